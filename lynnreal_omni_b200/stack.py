"""A stack of Flash-like W8A8 blocks over denoiser steps (the benchmark's config 4).

42 blocks of the config-2 block (``block.FlashBlockW8A8``; 24.4 GB of int8
weights per GPU, replicated), run for 3 denoiser steps on a latent of 64512
tokens sharded by contiguous token rows across the ranks, followed by one
all-gather of the bf16 output rows (``parallel.gather_rows``). Each (step,
block) uses its own adaLN table; the tables are precomputed, as the reference
caches them per timestep (model/fusion.py:145-162), so the timed work is the
W8A8 projection path only.
"""
from __future__ import annotations

import torch

from . import block as B
from . import workloads as W
from . import flash
from .parallel import gather_rows, shard_rows

LAYERS = 42
DENOISER_STEPS = 3
TOKENS = 64512


class FlashStackW8A8:
    def __init__(self, layers: int, device, seed: int = 0, hidden: int = W.HIDDEN, ffn: int = W.FFN,
                 text_dim: int = W.TEXT_DIM, steps: int = DENOISER_STEPS):
        self.blocks = [B.FlashBlockW8A8(B.make_weights(seed + 1000 * i, device, hidden, ffn, text_dim))
                       for i in range(layers)]
        g = W.generator(seed + 7, device)
        self.tables = [[(0.1 * torch.randn(1, 6 * hidden, generator=g, device=g.device)).to(torch.bfloat16)
                        for _ in range(layers)] for _ in range(steps)]
        self.steps = steps

    def forward(self, x_local: torch.Tensor, indices: torch.Tensor, context: torch.Tensor,
                ffn_events=None, compression: "Compression | None" = None) -> torch.Tensor:
        """x_local bf16 [1, m, D] (this rank's token rows) -> bf16 [1, m, D] after
        every denoiser step's pass through every block. ``ffn_events`` bracket
        the FFN-up GEMM of the first block of the first step. With
        ``compression``, blocks [start, end) of every step run on the kept rows
        and the residual is restored before block ``end`` (model/flash.py:65-84)."""
        h = x_local
        for s, step_tables in enumerate(self.tables):
            full = start_rows = None
            for i, (blk, table) in enumerate(zip(self.blocks, step_tables)):
                idx = indices
                if compression is not None:
                    if i == compression.start:
                        full = h
                        h = start_rows = flash.index_select(h, 1, compression.keep)
                    if i == compression.end:
                        h = flash.restore(full, h, start_rows, compression.inverse, compression.gain)
                    if compression.start <= i < compression.end:
                        idx = compression.indices(indices)
                h, _ = blk(h, table, idx, context, ffn_events=ffn_events if s == 0 and i == 0 else None)
        return h

    def launches_per_forward(self) -> int:
        return self.steps * len(self.blocks) * B.LAUNCHES_PER_FORWARD

    def sharded_forward(self, x_full_or_local, total_tokens: int, world: int, rank: int, indices, context,
                        gather: bool = True, ffn_events=None, compression: "Compression | None" = None,
                        bounds=None):
        """Run this rank's rows and all-gather the bf16 outputs ([total, D]);
        ``bounds`` are every rank's row blocks when they are not the default
        even split (frame-aligned shards for compression)."""
        local = x_full_or_local if x_full_or_local.shape[-2] != total_tokens else shard_rows(
            x_full_or_local, world, rank)
        out = self.forward(local.contiguous(), indices, context, ffn_events=ffn_events, compression=compression)
        if not gather or world == 1:
            return out
        return gather_rows(out.view(-1, out.shape[-1]), total_tokens, bounds=bounds)


class Compression:
    """Flash token compression of a video grid (frames x rows x columns,
    row-major rows): the kept rows and each row's restore source from
    ``flash.spatial_layout``; blocks [start, end) run compressed (the released
    schedule: 2 and 28 of 42)."""

    def __init__(self, frames: int, height: int, width: int, device, start: int = 2, end: int = 28,
                 gain: float = 1.0, first_frame: int = 0):
        t, h, w = torch.meshgrid(torch.arange(first_frame, first_frame + frames), torch.arange(height),
                                 torch.arange(width), indexing="ij")
        positions = torch.stack([t, h, w], -1).reshape(-1, 3).to(device)
        tags = torch.zeros(positions.shape[0], dtype=torch.int64, device=device)
        self.keep, self.inverse = flash.spatial_layout(positions, tags)
        self.start, self.end, self.gain = start, end, gain
        self._indices = {}

    def indices(self, indices: torch.Tensor) -> torch.Tensor:
        """adaLN indices of the kept rows (gathered once per indices tensor)."""
        key = (indices.data_ptr(), indices.numel(), indices._version, tuple(indices.stride()))
        if key not in self._indices:
            self._indices[key] = flash.index_select(indices, 0, self.keep)
        return self._indices[key]

    def kept_rows(self) -> int:
        return self.keep.numel()
