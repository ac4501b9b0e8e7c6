"""Element-wise fusion for the bf16 (non-quantised) block route.

Replaces model/elementwise_fusion.py: the block keeps its native RMSNorm,
modulation and attention modules and routes the two gated residuals and the
SwiGLU through the sm_100a kernels. Same functions, same call sequence
(model/elementwise_fusion.py:7-30), same rejection of ``fused_quant``.
"""
from __future__ import annotations

from types import MethodType

import torch.nn.functional as F

from .kernels import _gated_residual, _swiglu


def block_forward(self, hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None):
    """One DiT block: adaLN modulation table -> attention -> gated residual (slot 2)
    -> FFN (SwiGLU) -> gated residual (slot 5)."""
    linear = self.adaln_proj.linear
    width = self.adaln_proj.hidden_size
    table = linear(F.silu(temb).to(linear.weight.dtype)).view(-1, 6 * width)
    shift, scale, _, ff_shift, ff_scale, _ = table.chunk(6, dim=-1)

    def modulate(x, norm, s, b):
        return norm(x) * (1 + s.index_select(0, adaln_indices)) + b.index_select(0, adaln_indices)

    update = self.attn(modulate(hidden_states, self.norm1, scale, shift), rotary_emb, attention_mask)
    hidden_states = _gated_residual(hidden_states, update, table, adaln_indices, 2)
    projected = self.ff.net[0].proj(modulate(hidden_states, self.norm2, ff_scale, ff_shift))
    update = self.ff.net[2](_swiglu(projected))
    return _gated_residual(hidden_states, update, table, adaln_indices, 5)


def enable_elementwise_fusion(transformer, fused_quant=False):
    """Rebind every block's forward to ``block_forward``; evaluation-mode bf16 only."""
    if fused_quant or transformer.training:
        raise ValueError('elementwise fusion requires an evaluation-mode BF16 model')
    for block in transformer.transformer_blocks:
        block.forward = MethodType(block_forward, block)
    return dict(kind='elementwise', swiglu=True, gated_residual=True,
                normalization='native', attention_processor='native',
                blocks=len(transformer.transformer_blocks), activation_quantization_fused=False)
