"""INT8 tensor-core matmul with a fused scaled bf16 epilogue (sm_100a tcgen05).

Replaces model/int8_gemm.py. ``int8_matmul`` keeps the reference's signature,
contract check (ValueError) and allocation (a new bf16 [M, N] tensor) and
launches the tcgen05/TMEM/TMA kernel of liblr_w8a8.so on the current stream.
There is no autotuning and no fallback: the tile shape is fixed for B200
(128x256x128, persistent, double-buffered TMEM), operand layouts the tensor
memory accelerator cannot address run the library's CUDA-core kernel, whose
integer results are identical.

Extensions used by the B200 block (north-star items 2 and 4):
``int8_matmul_gelu`` (GELU-tanh fused into the epilogue) and
``int8_matmul_gated_residual`` (the gated residual of model/kernels.py:131-153
fused into the epilogue).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, ptr, stream_of

__all__ = ["int8_matmul", "int8_matmul_gelu", "int8_matmul_gated_residual", "int8_matmul_s32",
           "_torch_matmul"]

# Tile of the sm_100a kernel, in the reference's tile-tuple layout
# (BM, BN, BK, warps, stages, GROUP_M), model/int8_gemm.py:153-156.
TILE = (128, 256, 128, 6, 4, 8)


def _contract(a: torch.Tensor, b: torch.Tensor) -> None:
    # model/int8_gemm.py:97-98
    if a.dtype != torch.int8 or b.dtype != torch.int8 or not a.is_contiguous() or a.shape[1] != b.shape[0]:
        raise ValueError("INT8 GEMM requires contiguous row-major activations and compatible INT8 weights")
    if a.device.type != "cuda" or b.device != a.device:
        raise ValueError("INT8 GEMM requires CUDA tensors on one device")


def _scales(row_scale, column_scale, m: int, n: int):
    rs = row_scale.reshape(-1)
    cs = column_scale.reshape(-1)
    if rs.numel() != m or cs.numel() != n:
        raise ValueError(f"INT8 GEMM scales must have {m} rows and {n} columns")
    rs = rs.float().contiguous()
    cs = cs.float().contiguous()
    return rs, cs


def _launch(a, b, row_scale, column_scale, bias, epilogue, residual=None, table=None, indices=None,
            gate_slot=0, out=None, rows_to=None):
    _contract(a, b)
    m, k = a.shape
    n = b.shape[1]
    rs, cs = _scales(row_scale, column_scale, m, n)
    bb = None if bias is None else bias.to(torch.bfloat16).contiguous()
    if bb is not None and bb.numel() != n:
        raise ValueError("INT8 GEMM bias must have N elements")
    output = None if rows_to is not None else (
        torch.empty((m, n), device=a.device, dtype=torch.bfloat16) if out is None else out)
    resid_ptr, ldr, tbl, trows, twidth, idx, seq = None, 0, None, 0, 0, None, 1
    if epilogue == _lib.LR_EPI_GATED_RESIDUAL:
        res = residual.reshape(-1, residual.shape[-1])
        if res.shape != (m, n) or res.dtype != torch.bfloat16 or res.stride(1) != 1:
            raise ValueError("gated residual must be a bf16 [M, N] tensor with unit column stride")
        resid_ptr, ldr = ptr(res), res.stride(0)
        seq = residual.shape[-2] if residual.dim() >= 2 else 1
        if table is not None:
            if table.dtype != torch.bfloat16:
                raise ValueError("adaLN table must be bfloat16")
            tbl = table.contiguous()
            twidth = tbl.shape[-1]
            trows = tbl.numel() // twidth
            idx = indices.reshape(-1).to(torch.int64).contiguous()
            if idx.numel() < seq:
                raise ValueError(f"expected at least {seq} adaLN indices, got {idx.numel()}")
    lib = _lib.load()
    if rows_to is not None:
        ptrs, ld, row_offset = rows_to
        arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
        check(lib.lr_int8_gemm_rows_to(
            ptr(a), a.stride(0), ptr(b), b.stride(0), b.stride(1), m, n, k, ptr(rs), ptr(cs), ptr(bb), epilogue,
            resid_ptr, ldr, ptr(tbl), trows, twidth, ptr(idx), seq, gate_slot, arr, len(ptrs), ld, row_offset,
            stream_of(a)), "int8_matmul (rows to destinations)")
        return None
    ws_bytes = lib.lr_int8_gemm_workspace_bytes(m, n, k)
    # small-M shapes split K across the GPU: the int32 partial-sum workspace
    # comes from torch's caching allocator (the library allocates nothing)
    ws = torch.empty(ws_bytes // 4, device=a.device, dtype=torch.int32) if ws_bytes > 0 else None
    check(lib.lr_int8_gemm_ws(
        ptr(a), a.stride(0), ptr(b), b.stride(0), b.stride(1), m, n, k, ptr(rs), ptr(cs), ptr(bb),
        epilogue, resid_ptr, ldr, ptr(tbl), trows, twidth, ptr(idx), seq, gate_slot, ptr(output),
        output.stride(0), ptr(ws), ws_bytes, stream_of(a)), "int8_matmul")
    return output


def int8_matmul(a, b, row_scale, column_scale, bias=None, *, tile=None):
    """bf16((a @ b) * row_scale * column_scale + bias) with exact int32 accumulation.

    Replaces model/int8_gemm.py:96-163. a: int8 [M, K] contiguous; b: int8
    [K, N] with any strides (the reference's weights are the [K, N] view of a
    row-major [N, K] matrix); row_scale [M, 1]; column_scale [1, N]; bias bf16
    [N] or None. ``tile`` is accepted for signature compatibility; the sm_100a
    kernel has one tile shape (TILE).
    """
    if tile is not None and len(tuple(tile)) < 3:
        raise ValueError("tile must be a (BM, BN, BK, ...) tuple")
    return _launch(a, b, row_scale, column_scale, bias, _lib.LR_EPI_NONE)


def int8_matmul_gelu(a, b, row_scale, column_scale, bias=None):
    """``gelu_tanh(int8_matmul(...))`` in one kernel (GELU of the bf16 output, rounded to bf16)."""
    return _launch(a, b, row_scale, column_scale, bias, _lib.LR_EPI_GELU_TANH)


def int8_matmul_gated_residual(a, b, row_scale, column_scale, bias, residual, table, indices,
                               gate_slot, out=None, rows_to=None):
    """``_gated_residual(residual, int8_matmul(...), table, indices, gate_slot)`` in one kernel.

    Row r of the output uses table row ``indices[r % S]`` with S = residual.shape[-2];
    ``table=None`` means gate 1 (a plain bf16 residual add). ``out`` may be
    ``residual`` itself (in-place update of the residual stream).
    ``rows_to=(pointers, ld, row_offset)`` sends the output rows instead to row
    ``row_offset + r`` of each bf16 matrix at ``pointers`` (device addresses,
    possibly other GPUs' memory mapped by ``parallel.PeerRows``; leading
    dimension ``ld``) and returns None: the GEMM epilogue is the all-gather.
    """
    res_shape = residual.shape
    out2 = None if out is None else out.view(-1, out.shape[-1])
    y = _launch(a, b, row_scale, column_scale, bias, _lib.LR_EPI_GATED_RESIDUAL, residual, table,
                indices, gate_slot, out2, rows_to)
    return None if y is None else y.view(res_shape)


def int8_matmul_s32(a, b):
    """Raw int32 accumulators a @ b (exactness checks of the integer path)."""
    _contract(a, b)
    m, k = a.shape
    n = b.shape[1]
    acc = torch.empty((m, n), device=a.device, dtype=torch.int32)
    check(_lib.load().lr_int8_gemm_s32(ptr(a), a.stride(0), ptr(b), b.stride(0), b.stride(1), m, n, k,
                                       ptr(acc), stream_of(a)), "int8_matmul_s32")
    return acc


def _torch_matmul(a, b, row_scale, column_scale, bias):
    """The reference's cuBLASLt path (model/int8_gemm.py:84-92), kept as the
    integer known-answer comparator of ``int8_matmul``; never used as a fallback."""
    rows = a.shape[0]
    pad = max(32, -(-rows // 8) * 8) - rows
    flat = torch.nn.functional.pad(a, (0, 0, 0, pad)) if pad else a
    acc = torch._int_mm(flat, b)[:rows]
    output = acc.float() * row_scale.reshape(-1, 1).float() * column_scale.float()
    if bias is not None:
        output = output + bias.float()
    return output.to(torch.bfloat16)
