"""Attention core of the fused DiT block on the sm_100a tcgen05 kernel.

``attention_bshd(query, key, value)`` computes softmax(scale * Q K^T) V for
bf16 [B, S, H, 128] tensors (heads contiguous within a token; the strided
Q/K/V views of a fused QKV projection are used in place), fp32 scores and
softmax, bf16 output [B, S, H, 128]. It stands where FusedAttention calls
diffusers' attention dispatcher (model/fusion.py:55-57). Unsupported inputs
(a mask, another head size, another dtype) raise ValueError; torch's SDPA
remains available as ``fusion.sdpa_bshd`` for callers that need those.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import check, ptr, stream_of

__all__ = ["attention_bshd"]


def _token_view(t: torch.Tensor) -> torch.Tensor:
    """[B, S, H, D] with unit element stride, heads contiguous, batch stride =
    S * token stride and 16-byte aligned rows (what the kernel's TMA maps
    address), else a contiguous copy."""
    b, s, h, d = t.shape
    if (t.stride(3) == 1 and t.stride(2) == d and (b == 1 or t.stride(0) == s * t.stride(1))
            and t.stride(1) % 8 == 0 and t.data_ptr() % 16 == 0):
        return t
    return t.contiguous()


def attention_bshd(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, attn_mask=None,
                   scale: float | None = None) -> torch.Tensor:
    if attn_mask is not None:
        raise ValueError("attention_bshd: attention masks are not supported by the sm_100a kernel")
    for name, t in (("query", query), ("key", key), ("value", value)):
        if t.dtype != torch.bfloat16 or not t.is_cuda or t.ndim != 4:
            raise ValueError(f"attention_bshd: {name} must be a CUDA bf16 [B, S, H, D] tensor")
    b, sq, h, d = query.shape
    if key.shape[0] != b or key.shape[2:] != (h, d) or value.shape != key.shape:
        raise ValueError("attention_bshd: query/key/value shapes disagree")
    if d != 128:
        raise ValueError(f"attention_bshd: head_dim {d} (the kernel handles 128)")
    skv = key.shape[1]
    query, key, value = _token_view(query), _token_view(key), _token_view(value)
    out = torch.empty((b, sq, h, d), device=query.device, dtype=torch.bfloat16)
    sc = 1.0 / math.sqrt(d) if scale is None else float(scale)
    check(_lib.load().lr_attention_bf16(
        ptr(query), query.stride(1), ptr(key), key.stride(1), ptr(value), value.stride(1), b, sq, skv, h, d, sc,
        ptr(out), out.stride(1), stream_of(query)), "attention_bshd")
    return out
