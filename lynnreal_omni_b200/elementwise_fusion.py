"""Element-wise fusion for the bf16 (non-quantised) block route.

Replaces model/elementwise_fusion.py (:7-30): the block keeps its native
RMSNorm, modulation and attention modules and routes its two gated residuals
and its SwiGLU through the sm_100a kernels. The math is the reference's
(native norm, ``x * (1 + scale) + shift`` modulation in bf16, the same slots);
``enable_elementwise_fusion`` rejects ``fused_quant`` and training mode as the
reference does.
"""
from __future__ import annotations

from types import MethodType

from .fusion import resolve_adaln_table
from .kernels import _gated_residual, _swiglu


def _modulated(x, norm, rows, indices, shift_slot):
    """norm(x) * (1 + scale) + shift with the adaLN slots (shift_slot,
    shift_slot + 1) of each token's table row; bf16 torch arithmetic."""
    shift = rows[:, shift_slot].index_select(0, indices)
    scale = rows[:, shift_slot + 1].index_select(0, indices)
    return norm(x) * (1 + scale) + shift


def block_forward(self, hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None):
    """One DiT block: attention on the modulated input (slots 0, 1) -> gated
    residual (slot 2) -> SwiGLU FFN on the modulated residual (slots 3, 4) ->
    gated residual (slot 5)."""
    table = resolve_adaln_table(self, temb)
    rows = table.view(table.shape[0], 6, -1)  # [table rows, slot, hidden]
    attended = self.attn(_modulated(hidden_states, self.norm1, rows, adaln_indices, 0), rotary_emb, attention_mask)
    hidden_states = _gated_residual(hidden_states, attended, table, adaln_indices, 2)
    ffn_in = _modulated(hidden_states, self.norm2, rows, adaln_indices, 3)
    update = self.ff.net[2](_swiglu(self.ff.net[0].proj(ffn_in)))
    return _gated_residual(hidden_states, update, table, adaln_indices, 5)


def enable_elementwise_fusion(transformer, fused_quant=False):
    """Rebind every block's forward to ``block_forward``; evaluation-mode bf16 only."""
    if fused_quant or transformer.training:
        raise ValueError('elementwise fusion requires an evaluation-mode BF16 model')
    blocks = transformer.transformer_blocks
    for block in blocks:
        block.forward = MethodType(block_forward, block)
    return {"kind": "elementwise", "swiglu": True, "gated_residual": True, "normalization": "native",
            "attention_processor": "native", "blocks": len(blocks), "activation_quantization_fused": False}
