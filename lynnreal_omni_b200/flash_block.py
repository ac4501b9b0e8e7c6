"""A Flash DiT block at the release's shapes, run by ``fusion.fused_block``.

Shapes of the released Flash transformer's W8A8 projections (the GEMMs the
reference checks at install time, script/precompile.py:50): hidden 5376;
attention 56 heads x 128 with a fused QKV projection 5376 -> 21504 and the
output projection 7168 -> 5376; SwiGLU FFN 5376 -> 2 x 14336 -> 5376; per-head
RMSNorm of Q and K; adaLN modulation table [batch, 6 x 5376].

``FlashH3Block`` exposes exactly the attributes the reference's fused block
reads (model/fusion.py:12-98): ``adaln_proj`` (.linear, .hidden_size),
``norm1`` / ``norm2`` (.weight, .eps), ``attn`` (.to_qkv, .to_out, .norm_q,
.norm_k, .heads, .fused_projections, .set_processor, .processor) and
``ff.net[0].proj`` / ``ff.net[2]``; every projection is an ``Int8Linear`` with
random int8 weights and fp32 per-channel scales (as in config 0), so after
``fusion.enable_fusion(..., fused_quant=True)`` the whole block runs on this
package's kernels: the RMSNorm/adaLN/quant prologues, the INT8 GEMMs, the
Q/K RMSNorm+RoPE, the tcgen05 attention, SwiGLU+quant and the gated residuals.
The adaLN projection (a bf16 linear on the timestep embedding) is left to
torch; the benchmark passes a precomputed table, as the reference's
time-modulation cache does (model/fusion.py:145-162).
"""
from __future__ import annotations

from types import SimpleNamespace

import torch
from torch import nn

from . import workloads as W
from .int8 import Int8Linear

HIDDEN = 5376
HEADS = 56
HEAD_DIM = 128
FFN_INNER = 14336


def _int8_linear(n: int, k: int, gen: torch.Generator) -> Int8Linear:
    p = W.packed_linear(n, k, gen)
    return Int8Linear.from_packed(p.weight, p.scale, p.bias, gemm="triton")


class _Norm(nn.Module):
    def __init__(self, d: int, gen: torch.Generator, eps: float = 1e-6):
        super().__init__()
        w = (1 + 0.05 * torch.randn(d, generator=gen, device=gen.device)).to(torch.bfloat16)
        self.weight = nn.Parameter(w, requires_grad=False)
        self.eps = eps


class _Attention(nn.Module):
    def __init__(self, hidden: int, heads: int, gen: torch.Generator):
        super().__init__()
        inner = heads * HEAD_DIM
        self.heads = heads
        self.to_qkv = _int8_linear(3 * inner, hidden, gen)
        self.to_out = nn.ModuleList([_int8_linear(hidden, inner, gen), nn.Dropout(0.0)])
        self.norm_q, self.norm_k = _Norm(HEAD_DIM, gen), _Norm(HEAD_DIM, gen)
        self.fused_projections = True
        self.processor = None

    def set_processor(self, processor):
        self.processor = processor

    def forward(self, hidden_states, rotary_emb=None, attention_mask=None):
        return self.processor(self, hidden_states, rotary_emb, attention_mask)


class _Up(nn.Module):
    def __init__(self, proj: Int8Linear):
        super().__init__()
        self.proj = proj


class FlashH3Block(nn.Module):
    def __init__(self, seed: int = 0, device="cuda", hidden: int = HIDDEN, heads: int = HEADS,
                 ffn_inner: int = FFN_INNER):
        super().__init__()
        gen = W.generator(seed, device)
        adaln = nn.Linear(hidden, 6 * hidden, device=gen.device, dtype=torch.bfloat16)
        with torch.no_grad():
            adaln.weight.copy_(0.02 * torch.randn(adaln.weight.shape, generator=gen, device=gen.device))
            adaln.bias.copy_(0.02 * torch.randn(adaln.bias.shape, generator=gen, device=gen.device))
        self.adaln_linear = adaln
        self.adaln_proj = SimpleNamespace(linear=adaln, hidden_size=hidden)
        self.norm1, self.norm2 = _Norm(hidden, gen), _Norm(hidden, gen)
        self.attn = _Attention(hidden, heads, gen)
        self.ff = SimpleNamespace(net=nn.ModuleList([_Up(_int8_linear(2 * ffn_inner, hidden, gen)), nn.Dropout(0.0),
                                                     _int8_linear(hidden, ffn_inner, gen)]))
        self.ff_modules = self.ff.net


def make_inputs(tokens: int, seed: int = 1, device="cuda", hidden: int = HIDDEN):
    """Latent [1, tokens, hidden] ~N(0,1), timestep embedding, adaLN indices
    (one table row), rotary (cos, sin) [tokens, 128] of random phases."""
    gen = W.generator(seed, device)
    dev = gen.device
    x = torch.randn(1, tokens, hidden, generator=gen, device=dev).to(torch.bfloat16)
    temb = torch.randn(1, hidden, generator=gen, device=dev).to(torch.bfloat16)
    idx = torch.zeros(tokens, dtype=torch.int64, device=dev)
    phase = 10.0 * torch.rand(tokens, HEAD_DIM, generator=gen, device=dev)
    return x, temb, idx, (phase.cos(), phase.sin())


def ops_per_token(tokens: int, hidden: int = HIDDEN, heads: int = HEADS, ffn_inner: int = FFN_INNER):
    """(int8 GEMM ops, bf16 attention flops) per token of one block forward."""
    inner = heads * HEAD_DIM
    gemm = 2 * hidden * 3 * inner + 2 * inner * hidden + 2 * hidden * 2 * ffn_inner + 2 * ffn_inner * hidden
    attention = 4 * tokens * inner
    return gemm, attention
