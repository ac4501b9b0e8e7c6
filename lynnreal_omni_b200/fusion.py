"""Fused H3/Flash DiT block forward on the sm_100a kernels.

Replaces model/fusion.py: the block-level call sequence (``fused_block``,
model/fusion.py:61-98), the attention processor (``FusedAttention``, :12-58),
``enable_fusion`` (:118-142) and ``cache_time_modulation`` (:145-162). Which
kernels run, with which adaLN slots, in which order and under which
conditions is the reference's (it defines the numerics); the organisation of
the code is this package's: an adaLN-table resolver with its own per-timestep
cache, three block stages (attention input, FFN up-projection with the gated
residual, FFN down-projection) and an installer.

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

CACHE_ENTRIES = 16  # adaLN tables kept per block (oldest evicted first)


def sdpa_bshd(query, key, value, attn_mask=None):
    """Attention over [B, S, H, D] tensors with torch's SDPA."""
    out = F.scaled_dot_product_attention(query.transpose(1, 2), key.transpose(1, 2), value.transpose(1, 2),
                                         attn_mask=attn_mask, dropout_p=0.0, is_causal=False)
    return out.transpose(1, 2)


# ----------------------------------------------------------- adaLN tables
class _TimestepKey:
    """Forward pre-hook of a transformer: records the complete timestep tensor
    of the current forward as the adaLN-cache key every block reads."""

    def __init__(self):
        self.current = None

    def __call__(self, module, args, kwargs):
        if module.training or torch.is_grad_enabled():
            raise ValueError("cached time modulation requires frozen inference")
        times = kwargs["timestep"]
        self.current = (tuple(times.shape), str(times.dtype), tuple(times.detach().cpu().flatten().tolist()))


def resolve_adaln_table(block, temb, given=None):
    """The block's [rows, 6 * hidden] modulation table for this forward: the
    table passed in, else the block's cached one for the current timestep,
    else ``adaln_proj.linear(silu(temb))`` (cached when a key is active)."""
    if given is not None:
        return given
    cache = getattr(block, "_lynnreal_adaln_cache", None)
    key = block._lynnreal_cache_key.current if cache is not None else None
    if key is not None and key in cache:
        return cache[key]
    proj = block.adaln_proj
    table = proj.linear(F.silu(temb).to(proj.linear.weight.dtype)).view(-1, 6 * proj.hidden_size)
    if key is not None:
        while len(cache) >= CACHE_ENTRIES:
            del cache[next(iter(cache))]
        cache[key] = table
    return table


def cache_time_modulation(transformer):
    """Cache adaLN tables per complete timestep tensor (model/fusion.py:145-162)."""
    holder = _TimestepKey()
    blocks = transformer.transformer_blocks
    if any(not hasattr(block, "_lynnreal_fused_quant") for block in blocks):
        raise ValueError("time modulation caching requires fused blocks")
    for block in blocks:
        block._lynnreal_adaln_cache = {}
        block._lynnreal_cache_key = holder
    transformer.register_forward_pre_hook(holder, with_kwargs=True)
    return {"kind": "exact AdaLN tables", "key": "complete input noise-time tensor",
            "maximum_entries_per_block": CACHE_ENTRIES, "requires_immutable_weights": True}


# ------------------------------------------------------------- attention
class FusedAttention:
    """Attention processor: quantised QKV projection -> Q/K RMSNorm+RoPE ->
    attention -> W8A8 output projection (model/fusion.py:12-58)."""

    def __init__(self, original=None, ordered_qk=False, attention_fn=None):
        self.ordered_qk = ordered_qk
        self._attention_backend = getattr(original, "_attention_backend", None)
        self._parallel_config = getattr(original, "_parallel_config", None)
        self.attention_fn = attention_fn or attention_bshd

    @staticmethod
    def _projections(attn, hidden_states):
        if isinstance(hidden_states, tuple):  # int8 rows, row scales, shape from the fused prologue
            rows, scales, shape = hidden_states
            return attn.to_qkv.forward_quantized(rows, scales, shape[:-1]).chunk(3, dim=-1)
        if attn.fused_projections:
            return attn.to_qkv(hidden_states).chunk(3, dim=-1)
        return attn.to_q(hidden_states), attn.to_k(hidden_states), attn.to_v(hidden_states)

    def __call__(self, attn, hidden_states, rotary_emb=None, attention_mask=None):
        if rotary_emb is None or rotary_emb[0].ndim != 2:
            raise ValueError("fused attention requires a padless rotary layout")
        q, kk, v = (t.unflatten(-1, (attn.heads, -1)) for t in self._projections(attn, hidden_states))
        q, kk = k.qk_norm_rope(q, kk, attn.norm_q, attn.norm_k, rotary_emb)
        mixed = self.attention_fn(q, kk, v, attention_mask)
        return attn.to_out[1](attn.to_out[0](mixed.flatten(2, 3).type_as(q)))


# ------------------------------------------------------------ block stages
def _int8_capable(layer, fused_quant: bool) -> bool:
    return fused_quant and hasattr(layer, "forward_quantized")


def _attention_input(block, x, table, indices, fused_quant):
    """RMSNorm + adaLN (slots 0, 1) of the attention branch: int8 rows for a
    quantised QKV projection, bf16 otherwise."""
    if _int8_capable(block.attn.to_qkv, fused_quant):
        rows, scales = k._rms_adaln_quant_int8(x, block.norm1, table, indices, 0, 1)
        return rows, scales, x.shape
    return k._rms_adaln(x, block.norm1, table, indices, 0, 1)


def _ffn_up(block, x, attention_out, table, indices, fused_quant):
    """Gated residual of the attention branch (slot 2), RMSNorm + adaLN of the
    FFN branch (slots 3, 4) and the up-projection; returns (residual stream,
    projection)."""
    up = block.ff.net[0].proj
    if not _int8_capable(up, fused_quant):
        x = k._gated_residual(x, attention_out, table, indices, 2)
        return x, up(k._rms_adaln(x, block.norm2, table, indices, 3, 4))
    if block._lynnreal_residual_quant:
        x, rows, scales = k.residual_rms_quant(x, attention_out, block.norm2, table, indices)
    else:
        x = k._gated_residual(x, attention_out, table, indices, 2)
        rows, scales = k._rms_adaln_quant_int8(x, block.norm2, table, indices, 3, 4)
    return x, up.forward_quantized(rows, scales, x.shape[:-1])


def _ffn_down(down, projected, fused_quant):
    """SwiGLU (+ int8 quantisation) and the down-projection."""
    if _int8_capable(down, fused_quant):
        rows, scales = k._swiglu_quant_int8(projected)
        return down.forward_quantized(rows, scales, projected.shape[:-1])
    return down(k._swiglu(projected))


def fused_block(self, hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None, adaln_table=None):
    """One DiT block (model/fusion.py:61-98): adaLN table -> attention branch ->
    gated residual + FFN prologue -> FFN (SwiGLU) -> gated residual (slot 5)."""
    table = resolve_adaln_table(self, temb, adaln_table)
    quant = self._lynnreal_fused_quant
    attention_out = self.attn(_attention_input(self, hidden_states, table, adaln_indices, quant),
                              rotary_emb, attention_mask)
    residual, projected = _ffn_up(self, hidden_states, attention_out, table, adaln_indices, quant)
    return k._gated_residual(residual, _ffn_down(self.ff.net[2], projected, quant), table, adaln_indices, 5)


def guarded_block(self, *args, **kwargs):
    """The reference's guard swaps a failing block back to native math; here
    the native kernels are the only implementation, so errors propagate."""
    return fused_block(self, *args, **kwargs)


# -------------------------------------------------------------- installer
_DENSE_ONLY = ("h3_attention_token_stride", "h3_ffn_token_stride", "h3_depth_span")


def _modules(transformer):
    if hasattr(transformer, "modules"):
        return transformer.modules()
    return (m for block in transformer.transformer_blocks for m in block.modules())


def _install(block, fused_quant, residual_quant, processor):
    if any(getattr(block, name, 1) != 1 for name in _DENSE_ONLY):
        raise ValueError("fusion requires dense attention and FFN math within each block")
    block._lynnreal_fused_quant = fused_quant
    block._lynnreal_residual_quant = residual_quant
    if not hasattr(block, "_lynnreal_native_forward"):  # first installation keeps the native entry points
        block._lynnreal_native_forward = block.forward
        block._lynnreal_native_processor = getattr(block.attn, "processor", None)
    block.forward = MethodType(guarded_block, block)
    block.attn.set_processor(processor)


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
    blocks = transformer.transformer_blocks
    for block in blocks:
        _install(block, fused_quant, residual_quant,
                 FusedAttention(getattr(block.attn, "processor", None), ordered_qk, attention_fn))
    report = dict(rmsnorm_adaln=True, qk_norm_rope=True, swiglu=True,
                  qk_output_allocation="contiguous_without_copy", residual_block=1024, gated_residual=True)
    report.update(activation_quantization_fused=fused_quant, residual_ffn_norm_fused=residual_quant,
                  qk_ordered_reduction=ordered_qk, int8_epilogue_fused=fused_quant, blocks=len(blocks),
                  token_dropping=False)
    return report
