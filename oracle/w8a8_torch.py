"""Multi-threaded torch-CPU port of the W8A8 projection path.

TEST INFRASTRUCTURE ONLY (same rule as w8a8_oracle: imported by tests/,
__graft_entry__.smoke() and bench.py's CPU legs, never by the product).

This is the reference's own PyTorch (non-Triton) CPU implementation of the path,
restated for the benchmark's block: ``Int8Linear``'s torch path
(model/int8.py:41-68, quantiser :66-67, epilogue :55-58, ``torch._int_mm``) and
torch restatements of the Triton kernels (model/kernels.py), with the same
rounding points as w8a8_oracle. It runs on every host thread torch uses and is
checked bit-for-bit against w8a8_oracle in tests/test_oracle_torch.py.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16
F32 = torch.float32


def bf(x: torch.Tensor) -> torch.Tensor:
    """Round float32 to bf16 (nearest even) and back."""
    return x.to(BF16).to(F32)


def quantize_rows(x: torch.Tensor):
    """model/int8.py:66-67 / model/kernels.py:8-16 -> (int8, fp32 [rows, 1])."""
    x = x.to(F32)
    scale = x.abs().amax(-1, keepdim=True).clamp_min_(1e-8) / 127
    return (x / scale).round().clamp(-127, 127).to(torch.int8), scale


def int8_matmul(a: torch.Tensor, b_kn: torch.Tensor, row_scale, col_scale, bias=None) -> torch.Tensor:
    """Exact int32 GEMM + bf16 epilogue (model/int8_gemm.py:84-92) -> float32 (bf16 values)."""
    acc = torch._int_mm(a.contiguous(), b_kn)
    out = acc.to(F32) * row_scale.reshape(-1, 1).to(F32) * col_scale.reshape(1, -1).to(F32)
    if bias is not None:
        out = out + bias.to(F32)
    return bf(out)


def gelu_tanh_bf16(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x.to(BF16), approximate="tanh").to(F32)


def _thread_sums(v: torch.Tensor, threads: int, per_thread: int) -> torch.Tensor:
    rows, width = v.shape
    span = threads * per_thread
    reps = max(1, -(-width // span))
    padded = torch.zeros(rows, reps * span, dtype=F32)
    padded[:, :width] = v
    sq = (padded * padded).view(rows, reps, threads, per_thread)
    part = torch.zeros(rows, threads, dtype=F32)
    for r in range(reps):
        for e in range(per_thread):
            part = part + sq[:, r, :, e]
    return part


def _butterflies(part: torch.Tensor) -> torch.Tensor:
    rows, threads = part.shape
    warps = threads // 32
    lanes = part.view(rows, warps, 32)
    idx = torch.arange(32)
    for off in (16, 8, 4, 2, 1):
        lanes = lanes + lanes[:, :, idx ^ off]
    s = lanes[:, :, 0]
    off = warps // 2
    while off:
        s = s[:, :off] + s[:, off:2 * off]
        off //= 2
    return s[:, 0]


def sumsq_tree(v: torch.Tensor, threads: int = 256) -> torch.Tensor:
    """Row sum of squares in the bf16-output kernels' order (see w8a8_oracle.sumsq_tree)."""
    return _butterflies(_thread_sums(v, threads, 8))


def sumsq_quant(v: torch.Tensor) -> torch.Tensor:
    """The int8-output kernels' order (see w8a8_oracle.sumsq_quant)."""
    return _butterflies(_thread_sums(v, 256, 16 if v.shape[-1] > 2048 else 8))


def rms_adaln(x, weight, eps, table=None, indices=None, shift_slot=0, scale_slot=1, sequence=None,
              reduce=sumsq_tree):
    """RMSNorm + adaLN modulate (model/kernels.py:48-128) -> float32 (bf16 values)."""
    v = x.to(F32)
    rows, hidden = v.shape
    r = 1 / torch.sqrt(reduce(v) / hidden + torch.tensor(eps, dtype=F32))
    n = bf((v * r[:, None]) * weight.to(F32)[None, :])
    if table is None:
        return n
    seq = rows if sequence is None else sequence
    t = table.to(F32)[indices.reshape(-1)[torch.arange(rows) % seq]]
    shift = t[:, shift_slot * hidden:(shift_slot + 1) * hidden]
    scale = t[:, scale_slot * hidden:(scale_slot + 1) * hidden]
    return bf(bf(n * bf(1 + scale)) + shift)


def gated_residual(x, y, table=None, indices=None, gate_slot=0, sequence=None):
    """bf16(x + bf16(gate * y)) (model/kernels.py:131-153); table None -> gate 1."""
    x, y = x.to(F32), y.to(F32)
    if table is None:
        return bf(x + y)
    rows, hidden = x.shape
    seq = rows if sequence is None else sequence
    gate = table.to(F32)[indices.reshape(-1)[torch.arange(rows) % seq]][:, gate_slot * hidden:(gate_slot + 1) * hidden]
    return bf(x + bf(gate * y))


def flash_block(x, table, indices, context, w, reduce=sumsq_quant, stages=None, gelu_out=None):
    """The benchmark block's W8A8 path (lynnreal_omni_b200/block.py) on the CPU.

    x: bf16/fp32 [M, D]; w: a BlockWeights on the CPU. Returns (x' float32
    [M, D] of bf16 values, text K/V float32 [T, 2D]). The kernel order is the
    reference's fused block (model/fusion.py:61-98) with the benchmark's
    cross-attention and GELU FFN. ``stages`` (a dict), if given, receives the
    intermediates "attn", "cross" and "ffn_up" (the GELU-tanh output).
    ``gelu_out`` [M, FFN], if given, replaces this port's GELU-tanh output in
    the FFN-down step, so that step can be checked exactly against a device
    whose tanh differs in the last bit."""
    d = x.shape[-1]
    lin = lambda p, q, s: int8_matmul(q, p.weight.t(), s, p.scale, p.bias)  # noqa: E731
    h = x.to(F32)
    q, s = quantize_rows(rms_adaln(h, w.norm1, w.eps, table, indices, 0, 1, reduce=reduce))
    qkv = lin(w.qkv, q, s)
    q, s = quantize_rows(qkv[:, 2 * d:])
    h = gated_residual(h, lin(w.o, q, s), table, indices, 2)
    if stages is not None:
        stages["attn"] = h
    q, s = quantize_rows(rms_adaln(h, w.norm_cross, w.eps, reduce=reduce))
    cq = lin(w.cross_q, q, s)
    c8, cs = quantize_rows(context)
    kv = lin(w.cross_kv, c8, cs)
    q, s = quantize_rows(cq)
    h = gated_residual(h, lin(w.cross_o, q, s))
    if stages is not None:
        stages["cross"] = h
    q, s = quantize_rows(rms_adaln(h, w.norm2, w.eps, table, indices, 3, 4, reduce=reduce))
    u = gelu_tanh_bf16(lin(w.up, q, s))
    if stages is not None:
        stages["ffn_up"] = u
    q, s = quantize_rows(u if gelu_out is None else gelu_out.to(F32))
    h = gated_residual(h, lin(w.down, q, s), table, indices, 5)
    return h, kv
