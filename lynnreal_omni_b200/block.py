"""One Flash-like DiT block's W8A8 projection path (the benchmark's config 2).

Shapes: hidden D=6144 (48 heads x 128), fused QKV 6144->18432, O 6144->6144,
cross-attention Q/O 6144->6144 with text K/V 4096->2x6144 from a [512, 4096]
bf16 context, FFN 6144->24576 (GELU-tanh) ->6144. All projections are
``Int8Linear`` layers (int8 weights, fp32 per-channel scales, bf16 biases).

The call sequence follows the reference's fused block (model/fusion.py:61-98):
adaLN prologue kernel -> QKV projection -> attention -> O projection + gated
residual (slot 2) -> FFN prologue (slots 3, 4) -> FFN -> gated residual
(slot 5). Three differences, all outside the projection path:
  * the attention cores are stubs (the benchmark leaves them out of scope):
    self-attention returns V, cross-attention returns its query projection;
  * the benchmark's block has a cross-attention the reference's single-stream
    block lacks; its prologue is a slot-free RMSNorm + quantiser and its
    residual a plain add (gate 1);
  * the benchmark's FFN is GELU-tanh (fused into the up-projection epilogue)
    where the reference's is SwiGLU (``_swiglu_quant_int8``).
The gated residuals are fused into the O-proj / cross-O / FFN-down GEMM
epilogues (bit-identical to Int8Linear followed by ``_gated_residual``).
"""
from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace

import torch

from . import kernels as K
from . import workloads as W
from .int8 import Int8Linear
from .int8_gemm import int8_matmul_gated_residual, int8_matmul_gelu

# Launches of this package's kernels per forward (counted in forward()).
LAUNCHES_PER_FORWARD = 14


@dataclass
class BlockWeights:
    qkv: W.PackedLinear
    o: W.PackedLinear
    cross_q: W.PackedLinear
    cross_kv: W.PackedLinear
    cross_o: W.PackedLinear
    up: W.PackedLinear
    down: W.PackedLinear
    norm1: torch.Tensor
    norm2: torch.Tensor
    norm_cross: torch.Tensor
    eps: float = 1e-6


def make_weights(seed: int = 0, device="cpu", hidden: int = W.HIDDEN, ffn: int = W.FFN,
                 text_dim: int = W.TEXT_DIM) -> BlockWeights:
    """Random-init int8 weights as in config 0; norms ~N(1, 0.05) bf16."""
    g = W.generator(seed, device)
    dev = g.device
    lin = lambda n, k: W.packed_linear(n, k, g)  # noqa: E731
    norm = lambda: (1 + 0.05 * torch.randn(hidden, generator=g, device=dev)).to(torch.bfloat16)  # noqa: E731
    return BlockWeights(qkv=lin(3 * hidden, hidden), o=lin(hidden, hidden), cross_q=lin(hidden, hidden),
                        cross_kv=lin(2 * hidden, text_dim), cross_o=lin(hidden, hidden), up=lin(ffn, hidden),
                        down=lin(hidden, ffn), norm1=norm(), norm2=norm(), norm_cross=norm())


def make_inputs(tokens: int, seed: int, device="cpu", hidden: int = W.HIDDEN,
                text_tokens: int = W.TEXT_TOKENS, text_dim: int = W.TEXT_DIM):
    """Latent x bf16 [1, tokens, D] ~N(0,1); adaLN table bf16 [1, 6*D] ~N(0, 0.1)
    (the [B, 6, D] modulation viewed as rows); indices zeros [tokens]; text
    context bf16 [text_tokens, text_dim] ~N(0,1)."""
    g = W.generator(seed, device)
    dev = g.device
    x = torch.randn(1, tokens, hidden, generator=g, device=dev).to(torch.bfloat16)
    table = (0.1 * torch.randn(1, 6, hidden, generator=g, device=dev)).to(torch.bfloat16).view(1, 6 * hidden)
    idx = torch.zeros(tokens, dtype=torch.int64, device=dev)
    ctx = torch.randn(text_tokens, text_dim, generator=g, device=dev).to(torch.bfloat16)
    return x, table, idx, ctx


class FlashBlockW8A8:
    """The W8A8 path of one Flash-like block on the sm_100a kernels."""

    def __init__(self, weights: BlockWeights):
        mk = lambda p: Int8Linear.from_packed(p.weight, p.scale, p.bias, gemm="triton")  # noqa: E731
        self.qkv, self.o = mk(weights.qkv), mk(weights.o)
        self.cross_q, self.cross_kv, self.cross_o = mk(weights.cross_q), mk(weights.cross_kv), mk(weights.cross_o)
        self.up, self.down = mk(weights.up), mk(weights.down)
        self.norm1 = SimpleNamespace(weight=weights.norm1, eps=weights.eps)
        self.norm2 = SimpleNamespace(weight=weights.norm2, eps=weights.eps)
        self.norm_cross = SimpleNamespace(weight=weights.norm_cross, eps=weights.eps)
        self.hidden = weights.norm1.numel()

    @staticmethod
    def _gated(layer: Int8Linear, q, s, residual, table, idx, slot, out=None):
        return int8_matmul_gated_residual(q, layer.weight_int8, s, layer.weight_scale, layer.bias, residual,
                                          table, idx, slot, out=out)

    def forward(self, x, table, indices, context, ffn_events=None, probe=None, rows_to=None):
        """x bf16 [1, M, D] -> (x' bf16 [1, M, D], text K/V bf16 [T, 2D]).

        ``ffn_events`` (start, end) CUDA events, if given, bracket the FFN-up
        GEMM launch (the dominant kernel) on the current stream. ``probe``, if
        given, is called as ``probe(stage, tensor)`` with the block's
        intermediate results in stream order: "attn" (x after the O projection
        and its gated residual), "cross" (after the cross-attention residual),
        "ffn_up" (the GELU-tanh output [M, FFN]). The residual stream is then
        updated in place, so a probe that keeps a tensor must copy it.
        ``rows_to`` (pointers, ld, row_offset), if given, sends the block's
        output rows from the FFN-down GEMM epilogue to those destinations
        (``parallel.PeerRows``: every rank's gathered tensor) instead of the
        residual stream; the first result is then None.
        """
        d = self.hidden
        note = probe or (lambda stage, t: None)
        m = x.shape[-2]
        # self-attention: adaLN prologue (slots 0, 1) -> fused QKV
        q, s = K._rms_adaln_quant_int8(x, self.norm1, table, indices, 0, 1)
        qkv = self.qkv.forward_quantized(q, s, (m,))
        attn = qkv[:, 2 * d:]  # attention stub: output := V
        q, s = K.quantize_rows(attn)
        h = self._gated(self.o, q, s, x, table, indices, 2)  # O-proj + gated residual (slot 2)
        note("attn", h)
        # cross-attention: slot-free RMSNorm prologue -> Q; text K/V from the context
        q, s = K._rms_adaln_quant_int8(h, self.norm_cross, None, None, 0, 0)
        cq = self.cross_q.forward_quantized(q, s, (m,))
        cq8, cs = K.quantize_rows(context)
        kv = self.cross_kv.forward_quantized(cq8, cs, (context.shape[0],))
        q, s = K.quantize_rows(cq)  # cross-attention stub: output := its query projection
        self._gated(self.cross_o, q, s, h, None, None, 0, out=h)  # cross-O + plain residual, in place
        note("cross", h)
        # FFN: adaLN prologue (slots 3, 4) -> up + GELU-tanh -> quant -> down + gated residual (slot 5)
        q, s = K._rms_adaln_quant_int8(h, self.norm2, table, indices, 3, 4)
        if ffn_events is not None:
            ffn_events[0].record()
        u = int8_matmul_gelu(q, self.up.weight_int8, s, self.up.weight_scale, self.up.bias)
        if ffn_events is not None:
            ffn_events[1].record()
        note("ffn_up", u)
        q, s = K.quantize_rows(u)
        if rows_to is not None:
            int8_matmul_gated_residual(q, self.down.weight_int8, s, self.down.weight_scale, self.down.bias, h,
                                       table, indices, 5, rows_to=rows_to)
            return None, kv
        self._gated(self.down, q, s, h, table, indices, 5, out=h)
        return h, kv

    __call__ = forward
