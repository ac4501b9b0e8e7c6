"""Fused dense kernels of the W8A8 block path, on the sm_100a C ABI.

Same functions, arguments, return values and allocation behaviour as the
reference's model/kernels.py (each docstring cites the function it replaces);
the work runs in liblr_w8a8.so on the caller's current CUDA stream. Outputs are
freshly allocated on the input's device, inputs are made contiguous, and
contract violations raise ValueError. There is no other implementation behind
these functions: a missing library or a non-CUDA tensor is an error.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream_of

__all__ = [
    "quantize_rows", "int8_epilogue", "_rms_adaln", "_rms_adaln_quant_int8", "_gated_residual",
    "_swiglu", "_swiglu_quant_int8", "residual_rms_quant", "qk_norm_rope",
]


def _require_bf16(name: str, *tensors: torch.Tensor) -> None:
    for t in tensors:
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name}: expected bfloat16 tensors, got {t.dtype}")


def _adaln(table: torch.Tensor, indices: torch.Tensor, device: torch.device, sequence: int):
    """Contiguous table [rows, width] and flat int64 indices (model/kernels.py:262-263).

    Row r of the activations reads ``indices[r % sequence]``, so at least
    ``sequence`` indices are required."""
    table = table.contiguous()
    width = table.shape[-1]
    rows = table.numel() // width if width else 0
    idx = indices.reshape(-1)
    if idx.dtype != torch.int64:
        idx = idx.to(torch.int64)
    idx = idx.contiguous()
    if table.device != device or idx.device != device:
        raise ValueError("adaLN table and indices must be on the activations' device")
    if idx.numel() < sequence:
        raise ValueError(f"expected at least {sequence} adaLN indices, got {idx.numel()}")
    return table, rows, width, idx


def quantize_rows(value: torch.Tensor, *, arithmetic: str | None = None):
    """Per-row int8 quantisation -> (int8 [rows, width], fp32 [rows, 1]).

    Replaces model/kernels.py:19-24. Rows may be strided (unit column stride);
    e.g. a column slice of a fused QKV output is quantised in place.
    ``arithmetic`` (keyword only, not in the reference's signature) overrides
    the device's arithmetic mode for this call: "reference_gpu", "ieee" or
    "torch_cuda" (the reference's unfused PyTorch quantiser on a CUDA device,
    model/int8.py:66-67: scale = absmax x fl(1/127), IEEE quotient).
    """
    rows, width = value.shape
    _require_bf16("quantize_rows", value)
    if value.stride(1) != 1:
        value = value.contiguous()
    output = torch.empty((rows, width), device=value.device, dtype=torch.int8)
    scales = torch.empty(rows, 1, device=value.device, dtype=torch.float32)
    stride = value.stride(0) if rows > 1 else width
    if arithmetic is None:
        status = _lib.load().lr_quantize_rows(ptr(value), rows, width, stride, ptr(output), ptr(scales),
                                              stream_of(value))
    else:
        modes = dict(_lib.ARITHMETIC, torch_cuda=_lib.LR_ARITH_TORCH_CUDA)
        if arithmetic not in modes:
            raise ValueError(f"quantize_rows: arithmetic must be one of {sorted(modes)}, got {arithmetic!r}")
        status = _lib.load().lr_quantize_rows_arith(ptr(value), rows, width, stride, ptr(output), ptr(scales),
                                                    modes[arithmetic], stream_of(value))
    check(status, "quantize_rows")
    return output, scales


def int8_epilogue(accumulator, activation_scale, weight_scale, bias):
    """bf16((acc * activation_scale) * weight_scale + bias). Replaces model/kernels.py:41-46."""
    acc = accumulator.contiguous()
    if acc.dtype != torch.int32:
        raise ValueError("int8_epilogue: accumulator must be int32")
    cols = acc.shape[-1]
    rows = acc.numel() // cols if cols else 0
    rs = activation_scale.reshape(-1).float().contiguous()
    cs = weight_scale.reshape(-1).float().contiguous()
    if rs.numel() != rows or cs.numel() != cols:
        raise ValueError("int8_epilogue: scale shapes do not match the accumulator")
    b = None if bias is None else bias.to(torch.bfloat16).contiguous()
    output = torch.empty_like(acc, dtype=torch.bfloat16)
    check(_lib.load().lr_int8_epilogue(ptr(acc), rows, cols, ptr(rs), ptr(cs), ptr(b), ptr(output),
                                       stream_of(acc)), "int8_epilogue")
    return output


def _rms_common(source, norm, table, indices):
    source = source.contiguous()
    _require_bf16("rms_adaln", source, norm.weight)
    hidden = source.shape[-1]
    sequence = source.shape[-2] if source.dim() >= 2 else 1
    rows = source.numel() // hidden
    weight = norm.weight.contiguous()
    if weight.numel() != hidden:
        raise ValueError("rms_adaln: norm weight does not match the hidden size")
    if table is not None:
        _require_bf16("rms_adaln", table)
        table, trows, twidth, idx = _adaln(table, indices, source.device, sequence)
    else:
        trows, twidth, idx = 0, 0, None
    return source, hidden, sequence, rows, weight, table, trows, twidth, idx


def _rms_adaln(source, norm, table, indices, shift_slot, scale_slot):
    """RMSNorm + adaLN modulate -> bf16 like ``source``. Replaces model/kernels.py:260-272."""
    source, hidden, sequence, rows, weight, table, trows, twidth, idx = _rms_common(
        source, norm, table, indices)
    output = torch.empty_like(source)
    check(_lib.load().lr_rms_adaln(ptr(source), ptr(weight), float(norm.eps), ptr(table), trows, twidth,
                                   ptr(idx), sequence, rows, hidden, shift_slot, scale_slot, ptr(output),
                                   stream_of(source)), "_rms_adaln")
    return output


def _rms_adaln_quant_int8(source, norm, table, indices, shift_slot, scale_slot):
    """RMSNorm + adaLN modulate + row int8 quantisation -> (int8 [rows, hidden], fp32 [rows, 1]).

    Replaces model/kernels.py:275-289. ``table=None`` gives a plain RMSNorm + quantiser.
    """
    source, hidden, sequence, rows, weight, table, trows, twidth, idx = _rms_common(
        source, norm, table, indices)
    output = torch.empty((rows, hidden), device=source.device, dtype=torch.int8)
    scales = torch.empty((rows, 1), device=source.device, dtype=torch.float32)
    check(_lib.load().lr_rms_adaln_quant_int8(
        ptr(source), ptr(weight), float(norm.eps), ptr(table), trows, twidth, ptr(idx), sequence, rows,
        hidden, shift_slot, scale_slot, None, 0, None, ptr(output), ptr(scales), stream_of(source)),
        "_rms_adaln_quant_int8")
    return output, scales


def residual_rms_quant(source, update, norm, table, indices):
    """Gated residual (slot 2) + RMSNorm + adaLN (slots 3, 4) + quant in one pass
    -> (residual, int8, fp32). Replaces model/kernels.py:405-419."""
    source, hidden, sequence, rows, weight, table, trows, twidth, idx = _rms_common(
        source, norm, table, indices)
    update = update.contiguous()
    _require_bf16("residual_rms_quant", update)
    if update.shape != source.shape:
        raise ValueError("residual_rms_quant: update shape differs from source")
    residual = torch.empty_like(source)
    quantized = torch.empty((rows, hidden), device=source.device, dtype=torch.int8)
    scales = torch.empty((rows, 1), device=source.device, dtype=torch.float32)
    check(_lib.load().lr_rms_adaln_quant_int8(
        ptr(source), ptr(weight), float(norm.eps), ptr(table), trows, twidth, ptr(idx), sequence, rows,
        hidden, 3, 4, ptr(update), 2, ptr(residual), ptr(quantized), ptr(scales), stream_of(source)),
        "residual_rms_quant")
    return residual, quantized, scales


def _gated_residual(residual, update, table, indices, gate_slot):
    """bf16(residual + bf16(gate * update)). Replaces model/kernels.py:292-304."""
    residual = residual.contiguous()
    update = update.contiguous()
    _require_bf16("_gated_residual", residual, update)
    if update.shape != residual.shape:
        raise ValueError("_gated_residual: update shape differs from residual")
    hidden = residual.shape[-1]
    sequence = residual.shape[-2] if residual.dim() >= 2 else 1
    rows = residual.numel() // hidden
    if table is not None:
        _require_bf16("_gated_residual", table)
        table, trows, twidth, idx = _adaln(table, indices, residual.device, sequence)
    else:
        trows, twidth, idx = 0, 0, None
    output = torch.empty_like(residual)
    check(_lib.load().lr_gated_residual(ptr(residual), ptr(update), ptr(table), trows, twidth, ptr(idx),
                                        sequence, rows, hidden, gate_slot, ptr(output),
                                        stream_of(residual)), "_gated_residual")
    return output


def _swiglu(projected):
    """bf16(value * bf16(silu(gate))) over the last dim halves. Replaces model/kernels.py:307-315."""
    projected = projected.contiguous()
    _require_bf16("_swiglu", projected)
    inner = projected.shape[-1] // 2
    rows = projected.numel() // projected.shape[-1]
    output = torch.empty((*projected.shape[:-1], inner), device=projected.device, dtype=projected.dtype)
    check(_lib.load().lr_swiglu(ptr(projected), rows, inner, ptr(output), stream_of(projected)), "_swiglu")
    return output


def _swiglu_quant_int8(projected):
    """SwiGLU + row int8 quantisation -> (int8 [rows, inner], fp32 [rows, 1]).
    Replaces model/kernels.py:318-328."""
    projected = projected.contiguous()
    _require_bf16("_swiglu_quant_int8", projected)
    inner = projected.shape[-1] // 2
    rows = projected.numel() // projected.shape[-1]
    output = torch.empty((rows, inner), device=projected.device, dtype=torch.int8)
    scales = torch.empty((rows, 1), device=projected.device, dtype=torch.float32)
    check(_lib.load().lr_swiglu_quant_int8(ptr(projected), rows, inner, ptr(output), ptr(scales),
                                           stream_of(projected)), "_swiglu_quant_int8")
    return output, scales


def qk_norm_rope(query, key, norm_q, norm_k, rotary_emb):
    """Per-head RMSNorm + rotary embedding of Q and K -> contiguous (q_out, k_out).

    Replaces the launches of ``_qk_norm_full_rope_paired_kernel`` /
    ``_qk_norm_rope_kernel`` in FusedAttention (model/fusion.py:29-54).
    query, key: bf16 [B, S, H, D] (strided views of a fused QKV output are
    fine); norm_q/norm_k: modules with .weight (bf16 [D]) and .eps;
    rotary_emb: (cos, sin), each [S, rotary_dim].
    """
    cos, sin = rotary_emb
    if cos is None or cos.ndim != 2:
        raise ValueError("fused attention requires a padless rotary layout")
    b, s, h, d = query.shape
    rot = cos.shape[-1]
    if rot > d or rot % 2:
        raise ValueError("rotary dimensions must be even and fit the attention head")
    _require_bf16("qk_norm_rope", query, key, norm_q.weight, norm_k.weight)

    def layout(t):
        if t.stride(-1) != 1 or (b > 1 and t.stride(0) != s * t.stride(1)):
            t = t.contiguous()
        return t
    query, key = layout(query), layout(key)
    cos = cos.to(torch.float32).contiguous()
    sin = sin.to(torch.float32).contiguous()
    q_out = torch.empty((b, s, h, d), device=query.device, dtype=torch.bfloat16)
    k_out = torch.empty_like(q_out)
    check(_lib.load().lr_qk_norm_rope(
        ptr(query), ptr(key), query.stride(1), query.stride(2), key.stride(1), key.stride(2),
        ptr(norm_q.weight.contiguous()), ptr(norm_k.weight.contiguous()), ptr(cos), ptr(sin), b, s, h, d, rot,
        float(norm_q.eps), ptr(q_out), ptr(k_out), stream_of(query)), "qk_norm_rope")
    return q_out, k_out
