"""Fused H3/Flash DiT block forward on the sm_100a kernels.

Replaces model/fusion.py: the same block-level call sequence
(``fused_block``, model/fusion.py:61-98), attention processor
(``FusedAttention``, :12-58), ``enable_fusion`` (:118-142) and
``cache_time_modulation`` (:145-162), calling this package's kernels.

Differences, all deliberate:
  * no fallback: ``guarded_block`` does not swap a failing block back to the
    native diffusers math — a kernel error propagates;
  * ``residual_rms_quant`` (gated residual fused into the FFN prologue) is
    native on B200, so ``enable_fusion(fused_quant=True)`` uses it on every
    GPU instead of only on capability 9;
  * the Q/K RMSNorm+RoPE has one fixed reduction order, so the ``ordered_qk``
    option is accepted and has no effect;
  * the attention core is this package's tcgen05 kernel
    (``attention.attention_bshd``: bf16, head_dim 128, no mask) unless an
    ``attention_fn(q, k, v, attn_mask)`` taking [B, S, H, D] tensors is given
    (``sdpa_bshd`` for torch's SDPA, e.g. when a mask is needed, or diffusers'
    ``dispatch_attention_fn``).
"""
from __future__ import annotations

import os
from types import MethodType

import torch
import torch.nn.functional as F

from . import kernels as k
from .attention import attention_bshd


def sdpa_bshd(query, key, value, attn_mask=None):
    """Attention over [B, S, H, D] tensors with torch's SDPA."""
    out = F.scaled_dot_product_attention(query.transpose(1, 2), key.transpose(1, 2), value.transpose(1, 2),
                                         attn_mask=attn_mask, dropout_p=0.0, is_causal=False)
    return out.transpose(1, 2)


class FusedAttention:
    """Attention processor: quantised QKV projection -> Q/K RMSNorm+RoPE ->
    attention -> W8A8 output projection (model/fusion.py:12-58)."""

    def __init__(self, original=None, ordered_qk=False, attention_fn=None):
        self.ordered_qk = ordered_qk
        self._attention_backend = getattr(original, "_attention_backend", None)
        self._parallel_config = getattr(original, "_parallel_config", None)
        self.attention_fn = attention_fn or attention_bshd

    def __call__(self, attn, hidden_states, rotary_emb=None, attention_mask=None):
        if rotary_emb is None or rotary_emb[0].ndim != 2:
            raise ValueError("fused attention requires a padless rotary layout")
        if isinstance(hidden_states, tuple):
            quantized, scale, shape = hidden_states
            qkv = attn.to_qkv.forward_quantized(quantized, scale, shape[:-1])
            query, key, value = qkv.chunk(3, dim=-1)
        elif attn.fused_projections:
            query, key, value = attn.to_qkv(hidden_states).chunk(3, dim=-1)
        else:
            query, key, value = attn.to_q(hidden_states), attn.to_k(hidden_states), attn.to_v(hidden_states)
        query, key, value = [x.unflatten(-1, (attn.heads, -1)) for x in (query, key, value)]
        q_out, k_out = k.qk_norm_rope(query, key, attn.norm_q, attn.norm_k, rotary_emb)
        output = self.attention_fn(q_out, k_out, value, attention_mask)
        return attn.to_out[1](attn.to_out[0](output.flatten(2, 3).type_as(q_out)))


def fused_block(self, hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None, adaln_table=None):
    """One DiT block: adaLN table -> RMSNorm/adaLN/quant -> attention ->
    gated residual + FFN prologue -> FFN (SwiGLU) -> gated residual."""
    table = adaln_table
    cache = getattr(self, "_lynnreal_adaln_cache", None)
    key = self._lynnreal_cache_key[0] if cache is not None else None
    if table is None and key is not None:
        table = cache.get(key)
    if table is None:
        linear = self.adaln_proj.linear
        table = linear(F.silu(temb).to(linear.weight.dtype)).view(-1, 6 * self.adaln_proj.hidden_size)
        if key is not None:
            if len(cache) >= 16:
                cache.pop(next(iter(cache)))
            cache[key] = table
    use_quant = self._lynnreal_fused_quant
    if use_quant and hasattr(self.attn.to_qkv, "forward_quantized"):
        quantized, scales = k._rms_adaln_quant_int8(hidden_states, self.norm1, table, adaln_indices, 0, 1)
        attention_input = quantized, scales, hidden_states.shape
    else:
        attention_input = k._rms_adaln(hidden_states, self.norm1, table, adaln_indices, 0, 1)
    attention_output = self.attn(attention_input, rotary_emb, attention_mask)
    up, down = self.ff.net[0].proj, self.ff.net[2]
    if use_quant and hasattr(up, "forward_quantized"):
        if self._lynnreal_residual_quant:
            hidden_states, quantized, scales = k.residual_rms_quant(
                hidden_states, attention_output, self.norm2, table, adaln_indices)
        else:
            hidden_states = k._gated_residual(hidden_states, attention_output, table, adaln_indices, 2)
            quantized, scales = k._rms_adaln_quant_int8(hidden_states, self.norm2, table, adaln_indices, 3, 4)
        projected = up.forward_quantized(quantized, scales, hidden_states.shape[:-1])
    else:
        hidden_states = k._gated_residual(hidden_states, attention_output, table, adaln_indices, 2)
        projected = up(k._rms_adaln(hidden_states, self.norm2, table, adaln_indices, 3, 4))
    if use_quant and hasattr(down, "forward_quantized"):
        quantized, scales = k._swiglu_quant_int8(projected)
        output = down.forward_quantized(quantized, scales, projected.shape[:-1])
    else:
        output = down(k._swiglu(projected))
    return k._gated_residual(hidden_states, output, table, adaln_indices, 5)


def guarded_block(self, *args, **kwargs):
    """The reference's guard swaps a failing block back to native math; here
    the native kernels are the only implementation, so errors propagate."""
    return fused_block(self, *args, **kwargs)


def enable_fusion(transformer, fused_quant=False, attention_fn=None):
    """Route every block of ``transformer`` through ``fused_block``; returns the
    reference's report dict (model/fusion.py:118-142)."""
    residual_quant = bool(fused_quant)
    ordered_qk = residual_quant and os.environ.get("LYNNREAL_LONG_KERNELS", "1") != "0"
    if fused_quant:
        from .int8 import Int8Linear
        for module in _modules(transformer):
            if isinstance(module, Int8Linear):
                module.fused_ops = True
    for block in transformer.transformer_blocks:
        if any(getattr(block, name, 1) != 1 for name in ("h3_attention_token_stride", "h3_ffn_token_stride",
                                                         "h3_depth_span")):
            raise ValueError("fusion requires dense attention and FFN math within each block")
        block._lynnreal_fused_quant = fused_quant
        block._lynnreal_residual_quant = residual_quant
        if not hasattr(block, "_lynnreal_native_forward"):
            block._lynnreal_native_forward = block.forward
            block._lynnreal_native_processor = getattr(block.attn, "processor", None)
        block.forward = MethodType(guarded_block, block)
        block.attn.set_processor(FusedAttention(getattr(block.attn, "processor", None), ordered_qk, attention_fn))
    return {"rmsnorm_adaln": True, "qk_norm_rope": True, "swiglu": True,
            "qk_output_allocation": "contiguous_without_copy", "residual_block": 1024,
            "gated_residual": True, "activation_quantization_fused": fused_quant,
            "residual_ffn_norm_fused": residual_quant,
            "qk_ordered_reduction": ordered_qk,
            "int8_epilogue_fused": fused_quant,
            "blocks": len(transformer.transformer_blocks), "token_dropping": False}


def _modules(transformer):
    if hasattr(transformer, "modules"):
        return transformer.modules()
    return (m for block in transformer.transformer_blocks for m in block.modules())


def cache_time_modulation(transformer):
    """Cache adaLN tables per complete timestep tensor (model/fusion.py:145-162)."""
    key = [None]
    for block in transformer.transformer_blocks:
        if not hasattr(block, "_lynnreal_fused_quant"):
            raise ValueError("time modulation caching requires fused blocks")
        block._lynnreal_adaln_cache = {}
        block._lynnreal_cache_key = key

    def select_key(module, args, kwargs):
        if module.training or torch.is_grad_enabled():
            raise ValueError("cached time modulation requires frozen inference")
        times = kwargs["timestep"]
        key[0] = (tuple(times.shape), str(times.dtype), tuple(times.detach().cpu().flatten().tolist()))

    transformer.register_forward_pre_hook(select_key, with_kwargs=True)
    return {"kind": "exact AdaLN tables", "key": "complete input noise-time tensor",
            "maximum_entries_per_block": 16, "requires_immutable_weights": True}
