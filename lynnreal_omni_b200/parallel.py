"""Token-row sharding across GPUs and the final output all-gather.

The projection path is independent per token row, so a latent of M rows is
split into contiguous per-rank row blocks, every rank runs the W8A8 path on its
block with the int8 weights replicated, and the only collective is one
all-gather of the bf16 output rows at the end (NCCL over NVLink/NVSwitch on a
B200 node). Shards differ by at most one row; the gather pads every shard to
the largest one and strips the padding afterwards.

``PeerRows`` replaces that collective where the last projection of the path
can write its rows itself: every rank's copy of the gathered tensor is mapped
into every other rank (CUDA IPC, peer access over NVLink), and the projection's
GEMM epilogue stores each output tile into all of them
(``int8_matmul_gated_residual(..., rows_to=...)``), so the transfer overlaps
the tensor-core work instead of following it.
"""
from __future__ import annotations

import ctypes

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


class RowGather:
    """All-gather of every rank's row block into the full ``[total, ...]`` tensor.

    Built once per (total, bounds): equal shards (12240 rows over 1/2/4/8 GPUs,
    for instance) are gathered straight from ``local`` into the output with one
    ``all_gather_into_tensor``; unequal shards go through a padded staging
    buffer and are compacted afterwards. ``out``, if given, receives the rows
    (equal shards only need no copy at all).
    """

    def __init__(self, total: int, group=None, bounds=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.total = total
        self.bounds = bounds or [shard_bounds(total, self.world, r) for r in range(self.world)]
        b = self.bounds
        if len(b) != self.world or b[0][0] != 0 or b[-1][1] != total or any(
                b[r][1] != b[r + 1][0] for r in range(self.world - 1)):
            raise ValueError("row bounds must tile [0, total) in rank order")
        self.width = max(e - s for s, e in b)
        self.even = all(e - s == self.width for s, e in b)

    def __call__(self, local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        start, stop = self.bounds[self.rank]
        if local.shape[0] != stop - start:
            raise ValueError(f"rank {self.rank} holds {local.shape[0]} rows, expected {stop - start}")
        shape = (self.total, *local.shape[1:])
        if out is not None and (tuple(out.shape) != shape or out.dtype != local.dtype or not out.is_contiguous()):
            raise ValueError(f"gather output must be a contiguous {local.dtype} tensor of shape {shape}")
        if self.even:
            out = local.new_empty(shape) if out is None else out
            dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
            return out
        padded = local.new_zeros((self.width, *local.shape[1:]))
        padded[: local.shape[0]] = local
        staged = local.new_empty((self.world * self.width, *local.shape[1:]))
        dist.all_gather_into_tensor(staged, padded, group=self.group)
        parts = [staged[r * self.width: r * self.width + (e - s)] for r, (s, e) in enumerate(self.bounds)]
        if out is None:
            return torch.cat(parts, dim=0)
        return torch.cat(parts, dim=0, out=out)


def gather_rows(local: torch.Tensor, total: int, group=None, bounds=None) -> torch.Tensor:
    """All-gather the row blocks of every rank into the full [total, ...] tensor.

    ``local`` is this rank's block (rows on dim 0); ``bounds[r]`` is rank r's
    [start, stop) (default: ``shard_bounds``). The result is identical on every
    rank (see ``RowGather``).
    """
    return RowGather(total, group, bounds)(local)


class PeerRows:
    """Gathered ``[total, width]`` bf16 tensors that a GEMM epilogue fills on
    every rank at once.

    Each rank allocates ``buffers`` such tensors, exports their CUDA IPC
    handles and maps every other rank's, so ``destinations(i)`` lists the
    device addresses of buffer ``i`` on all ranks (rank order), usable as the
    ``rows_to`` pointers of ``int8_gemm`` calls; this rank's rows start at
    ``row_offset``. Buffers alternate between steps so that one step's rows
    can be read while the next is written. ``barrier()`` is a stream-ordered
    cross-GPU barrier (an NCCL all-reduce of one element on the current
    stream): once it has run on every rank after the writing kernels, all
    ranks' rows are visible; before the next write into a buffer it also
    tells every writer that its readers are done with it.
    """

    def __init__(self, total: int, width: int, device, group=None, buffers: int = 2):
        from . import _lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.total, self.width = total, width
        start, stop = shard_bounds(total, self.world, self.rank)
        self.row_offset, self.rows = start, stop - start
        self.lib = _lib.load()
        self.local = [torch.empty(total, width, dtype=torch.bfloat16, device=device) for _ in range(buffers)]
        exported = []
        for t in self.local:
            handle = ctypes.create_string_buffer(64)
            offset = ctypes.c_int64(0)
            _lib.check(self.lib.lr_ipc_export(t.data_ptr(), handle, ctypes.byref(offset)), "PeerRows: export")
            exported.append((handle.raw, offset.value))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, exported, group=group)
        self.mapped = []  # (pointer, offset) of every imported peer buffer, for release
        self.pointers = []
        for i in range(buffers):
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(self.local[i].data_ptr())
                    continue
                raw, offset = everyone[r][i]
                out = ctypes.c_void_p(0)
                _lib.check(self.lib.lr_ipc_import(raw, offset, ctypes.byref(out)), "PeerRows: import")
                self.mapped.append((out.value, offset))
                ptrs.append(out.value)
            self.pointers.append(ptrs)
        self._flag = torch.zeros(1, dtype=torch.int32, device=device)

    def destinations(self, slot: int):
        """``rows_to`` argument for buffer ``slot``: (pointers, ld, row_offset)."""
        return self.pointers[slot], self.width, self.row_offset

    def barrier(self) -> None:
        dist.all_reduce(self._flag, group=self.group)

    def close(self) -> None:
        from . import _lib
        for p, offset in self.mapped:
            _lib.check(self.lib.lr_ipc_release(p, offset), "PeerRows: release")
        self.mapped.clear()
        self.pointers.clear()
