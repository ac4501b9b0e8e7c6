"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

There is no public dataset on this path: every config is synthetic.
  c0  one W8A8 linear: x bf16 [1024, 6144] ~N(0,1) with 0.5% of the channels
      scaled x20, W int8 [6144, 6144] uniform in [-127, 127], per-channel fp32
      scales ~U(0.5e-3, 2e-3), bf16 bias ~N(0, 0.02)
  c1  block prologue: x bf16 [1, 12240, 6144] ~N(0,1), RMSNorm weight ~N(1, 0.05),
      eps 1e-6, modulation bf16 [1, 6, 6144] ~N(0, 0.1), y bf16 ~N(0,1)
  c2  one Flash-like DiT block at M=12240, D=6144 (see block.py)
  c3  GEMM sweep M x (K, N)
Generation runs on the CPU with ``torch.Generator().manual_seed(seed)`` unless a
CUDA generator is asked for (large bench tensors), so CPU-generated inputs are
identical on every machine with this torch build.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

HIDDEN = 6144
HEADS = 48
HEAD_DIM = 128
FFN = 24576
TEXT_TOKENS = 512
TEXT_DIM = 4096
BLOCK_TOKENS = 12240  # 22-frame 540p latent
SWEEP_M = (256, 2048, 12240, 32768, 64512)
SWEEP_KN = ((6144, 6144), (6144, 18432), (6144, 24576), (24576, 6144))


def generator(seed: int, device: str | torch.device = "cpu") -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def activations(m: int, k: int, gen: torch.Generator, outlier_frac: float = 0.005,
                outlier_scale: float = 20.0, device=None) -> torch.Tensor:
    """bf16 [m, k] ~N(0,1) with a seeded fraction of channels scaled as outliers."""
    device = device or gen.device
    x = torch.randn(m, k, generator=gen, device=device)
    count = max(1, round(outlier_frac * k)) if outlier_frac > 0 else 0
    if count:
        cols = torch.randperm(k, generator=gen, device=device)[:count]
        x[:, cols] *= outlier_scale
    return x.to(torch.bfloat16)


@dataclass
class PackedLinear:
    """A W8A8 projection in the reference's packed layout (model/flash_int8.py:36):
    int8 weight [out, in], fp32 scale [out, 1], bf16 bias [out] or None."""
    weight: torch.Tensor
    scale: torch.Tensor
    bias: torch.Tensor | None

    def to(self, device) -> "PackedLinear":
        return PackedLinear(self.weight.to(device), self.scale.to(device),
                            None if self.bias is None else self.bias.to(device))


def packed_linear(n: int, k: int, gen: torch.Generator, bias: bool = True, device=None) -> PackedLinear:
    """int8 W [n, k] uniform in [-127, 127]; scales ~U(0.5e-3, 2e-3); bias ~N(0, 0.02)."""
    device = device or gen.device
    w = torch.randint(-127, 128, (n, k), generator=gen, device=device, dtype=torch.int8)
    s = torch.empty(n, 1, device=device).uniform_(0.5e-3, 2e-3, generator=gen)
    b = (torch.randn(n, generator=gen, device=device) * 0.02).to(torch.bfloat16) if bias else None
    return PackedLinear(w, s, b)


def config0(seed: int = 0, m: int = 1024, k: int = HIDDEN, n: int = HIDDEN):
    """c0: (x bf16 [m, k], PackedLinear [n, k])."""
    g = generator(seed)
    x = activations(m, k, g)
    return x, packed_linear(n, k, g)


@dataclass
class Prologue:
    x: torch.Tensor        # bf16 [1, M, D]
    y: torch.Tensor        # bf16 [1, M, D] (the update of the gated residual)
    norm_weight: torch.Tensor  # bf16 [D]
    eps: float
    table: torch.Tensor    # bf16 [1, 6*D]  (the [B, 6, D] modulation viewed as rows)
    indices: torch.Tensor  # int64 [M]


def config1(seed: int = 0, m: int = BLOCK_TOKENS, d: int = HIDDEN, device=None) -> Prologue:
    g = generator(seed) if device is None else generator(seed, device)
    dev = g.device
    x = torch.randn(1, m, d, generator=g, device=dev).to(torch.bfloat16)
    y = torch.randn(1, m, d, generator=g, device=dev).to(torch.bfloat16)
    w = (1.0 + 0.05 * torch.randn(d, generator=g, device=dev)).to(torch.bfloat16)
    table = (0.1 * torch.randn(1, 6, d, generator=g, device=dev)).to(torch.bfloat16).view(1, 6 * d)
    idx = torch.zeros(m, dtype=torch.int64, device=dev)
    return Prologue(x, y, w, 1e-6, table, idx)


def gemm_operands(m: int, k: int, n: int, seed: int = 219, device=None, bias: bool = False):
    """Operands in the style of the reference's install-time GEMM check
    (script/precompile.py:56-59): int8 A [m, k], B = [n, k] int8 transposed to
    a [k, n] view, row scales rand/127 [m, 1], column scales rand/127 [1, n]."""
    g = generator(seed) if device is None else generator(seed, device)
    dev = g.device
    a = torch.randint(-127, 128, (m, k), generator=g, device=dev, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8).t()
    rs = torch.rand(m, 1, generator=g, device=dev) / 127
    cs = torch.rand(1, n, generator=g, device=dev) / 127
    bb = (torch.randn(n, generator=g, device=dev) * 0.02).to(torch.bfloat16) if bias else None
    return a, b, rs, cs, bb
