"""CPU oracle of the LynnReal-Omni W8A8 projection path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py`` (its CPU-baseline leg and its ``--impl reference`` arm) may import
this module; the product path never does, and nothing here runs on a GPU.

Each function restates one function of the reference (file:line cited; paths
are relative to the reference project root) as plain CPU arithmetic:
  * element-wise and row work in numpy float32, every product and sum rounded
    on its own (the reference launches with ``enable_fp_fusion=False``), with
    the reference's bf16 rounding points written out as ``bf16_round``;
  * the integer GEMM through ``torch._int_mm`` on the CPU (exact int32), the
    same library call the reference's own torch path makes.

Reduction order. The only order-dependent quantity on the path is the
RMSNorm sum of squares. ``sumsq_numpy`` is the order of the reference's Triton
kernel when run by the Triton interpreter (``np.sum``); ``sumsq_tree`` is the
fixed tree of the CUDA kernels (256 threads x 8-column chunks added in order,
then a warp butterfly, then a butterfly over the 8 warps), which is also the
order of the reference's kernel compiled for the GPU. All other steps are
order-independent.

Division and square root are IEEE round-to-nearest here, as in the
reference's PyTorch path and under the Triton interpreter. The CUDA kernels
compute them that way in their "ieee" arithmetic mode; their default mode uses
the approximate instructions the reference's kernels compile to on the GPU,
which no CPU restatement reproduces bit for bit.

Parity pinning: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``: the reference's torch path and its Triton
kernels under the Triton interpreter).
"""
from __future__ import annotations

import numpy as np
import torch

F32 = np.float32

# ---------------------------------------------------------------- bf16 helpers


def bf16_bits(x) -> np.ndarray:
    """Round float32 values to bf16 (nearest, ties to even); return uint16 bits."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    if nan.any():
        rounded = np.where(nan, (u >> 16) | 0x40, rounded)
    return rounded.astype(np.uint16)


def from_bf16_bits(bits) -> np.ndarray:
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(F32)


def bf16_round(x) -> np.ndarray:
    """bf(x): round to bf16 and back to float32."""
    return from_bf16_bits(bf16_bits(x))


def to_numpy_f32(t: torch.Tensor) -> np.ndarray:
    """bf16/fp32 torch tensor -> float32 numpy array (exact)."""
    return t.detach().to("cpu", torch.float32).contiguous().numpy()


def to_torch_bf16(x: np.ndarray) -> torch.Tensor:
    """float32 array of bf16-representable values -> bf16 torch tensor (exact)."""
    bits = bf16_bits(x)
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)


# ------------------------------------------------------------ K1 row quantiser


def quantize_rows(x):
    """Per-row symmetric int8 quantisation.

    model/kernels.py:8-16 (``_quantize_rows_kernel``) and model/int8.py:66-67:
    scale = max(max|x|, 1e-8) / 127 ; q = round_half_even(clamp(x / scale, -127, 127)).
    Returns (int8 [rows, width], float32 [rows, 1]).
    """
    x = np.asarray(x, dtype=F32)
    amax = np.max(np.abs(x), axis=-1, keepdims=True) if x.shape[-1] else np.zeros(x.shape[:-1] + (1,), F32)
    scale = (np.maximum(amax, F32(1e-8)) / F32(127)).astype(F32)
    q = np.rint(np.clip(x / scale, F32(-127), F32(127))).astype(np.int8)
    return q, scale


# ------------------------------------------------------- K10 GEMM + K2 epilogue


def int8_gemm_s32(a: np.ndarray, b_kn: np.ndarray) -> np.ndarray:
    """Exact int32 accumulators acc = a @ b (model/int8_gemm.py:88; model/int8.py:51)."""
    at = torch.from_numpy(np.ascontiguousarray(a, dtype=np.int8))
    bt = torch.from_numpy(np.ascontiguousarray(b_kn, dtype=np.int8))
    return torch._int_mm(at, bt).numpy()


def int8_epilogue(acc, row_scale, col_scale, bias=None) -> np.ndarray:
    """bf16((float(acc) * row_scale) * col_scale + bias) as float32.

    model/kernels.py:27-38 (``_int8_epilogue_kernel``), model/int8_gemm.py:84-92
    (``_torch_matmul``), model/int8.py:55-58.
    """
    out = np.asarray(acc).astype(F32) * np.asarray(row_scale, F32).reshape(-1, 1)
    out = out * np.asarray(col_scale, F32).reshape(1, -1)
    if bias is not None:
        out = out + np.asarray(bias, F32).reshape(1, -1)
    return bf16_round(out)


def int8_matmul(a, b_kn, row_scale, col_scale, bias=None) -> np.ndarray:
    """INT8 GEMM with the fused bf16 epilogue (model/int8_gemm.py:13-46, 84-92)."""
    return int8_epilogue(int8_gemm_s32(a, b_kn), row_scale, col_scale, bias)


def gelu_tanh_bf16(x) -> np.ndarray:
    """tanh-approximated GELU of bf16 values, result rounded to bf16.

    The reference has no GELU; this is the module semantics of a bf16
    ``Int8Linear`` output fed to ``torch.nn.functional.gelu(approximate="tanh")``.
    """
    t = to_torch_bf16(np.asarray(x, F32))
    return to_numpy_f32(torch.nn.functional.gelu(t, approximate="tanh"))


def int8_matmul_gelu(a, b_kn, row_scale, col_scale, bias=None) -> np.ndarray:
    return gelu_tanh_bf16(int8_matmul(a, b_kn, row_scale, col_scale, bias))


def int8_matmul_gated_residual(a, b_kn, row_scale, col_scale, bias, residual, table, indices,
                               gate_slot) -> np.ndarray:
    """Int8Linear output followed by the gated residual (model/int8.py:41-58 then
    model/kernels.py:131-153): bf16(x + bf16(gate * bf16(dequant)))."""
    y = int8_matmul(a, b_kn, row_scale, col_scale, bias)
    return gated_residual(residual, y, table, indices, gate_slot)


# ------------------------------------------------------------ reductions


def sumsq_numpy(v: np.ndarray) -> np.ndarray:
    """Row sum of squares in the order of the reference kernel run by the Triton
    interpreter: ``np.sum`` over the kernel's power-of-two block
    (``triton.next_power_of_2(hidden)``, model/kernels.py:270,287), zero padded."""
    v = np.asarray(v, F32)
    rows, width = v.shape
    block = 1 << max(0, (width - 1).bit_length())
    padded = np.zeros((rows, block), F32)
    padded[:, :width] = v
    return np.sum(padded * padded, axis=-1, dtype=F32)


def _thread_sums(v: np.ndarray, threads: int, per_thread: int) -> np.ndarray:
    """[rows, threads] sums of squares: thread t adds the squares of columns
    (r*threads + t)*per_thread + e, e = 0..per_thread-1, r = 0, 1, ... in order."""
    v = np.asarray(v, F32)
    rows, width = v.shape
    span = threads * per_thread
    reps = max(1, -(-width // span))
    padded = np.zeros((rows, reps * span), F32)
    padded[:, :width] = v
    sq = (padded * padded).reshape(rows, reps, threads, per_thread)
    part = np.zeros((rows, threads), F32)
    for r in range(reps):
        for e in range(per_thread):
            part = part + sq[:, r, :, e]
    return part


def _butterflies(part: np.ndarray) -> np.ndarray:
    """An xor butterfly (16, 8, 4, 2, 1) over the 32 lanes of each warp, then
    one over the warp sums as the lanes of one warp would run it
    (8 warps: ((w0 + w4) + (w2 + w6)) + ((w1 + w5) + (w3 + w7)))."""
    rows, threads = part.shape
    warps = threads // 32
    lanes = part.reshape(rows, warps, 32)
    idx = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        lanes = lanes + lanes[:, :, idx ^ off]
    s = lanes[:, :, 0]
    off = warps // 2
    while off:
        s = s[:, :off] + s[:, off:2 * off]
        off //= 2
    return s[:, 0]


def sumsq_tree(v: np.ndarray, threads: int = 256) -> np.ndarray:
    """Row sum of squares in the order of the CUDA kernels with bf16 output
    (K3), which is the order of the reference's compiled ``tl.sum`` in its
    bf16-output kernel (model/kernels.py:65; 8 warps, 8 columns per thread
    from the 16-byte bf16 accesses) for rows of 2048 columns or more: each
    thread adds its columns in order, then ``_butterflies``."""
    return _butterflies(_thread_sums(v, threads, 8))


def sumsq_tree16(v: np.ndarray, threads: int = 256) -> np.ndarray:
    """Row sum of squares in the order of the reference's compiled int8-output
    kernels (model/kernels.py:106; their 16-byte int8 stores lay a row out
    with 16 columns per thread: thread t adds columns 4096 r + 16 t + e in
    order), then ``_butterflies``; the CUDA K4/K8 kernels reproduce it."""
    return _butterflies(_thread_sums(v, threads, 16))


def sumsq_quant(v: np.ndarray) -> np.ndarray:
    """The order of the int8-output RMSNorm kernels: 16 columns per thread for
    rows of more than 2048 columns (a 4096-column block or larger), else 8."""
    return sumsq_tree16(v) if np.asarray(v).shape[-1] > 2048 else sumsq_tree(v)


# --------------------------------------------------- K3 / K4 / K8 row kernels


def _table_rows(table, indices, rows: int, sequence: int):
    table = np.asarray(table, F32)
    idx = np.asarray(indices, np.int64).reshape(-1)
    return table[idx[np.arange(rows) % sequence]]


def _rms_modulate(v, weight, eps, table, indices, sequence, shift_slot, scale_slot, reduce):
    rows, hidden = v.shape
    ss = reduce(v)
    r = (F32(1) / np.sqrt(ss / F32(hidden) + F32(eps))).astype(F32)
    n = bf16_round((v * r[:, None]) * np.asarray(weight, F32)[None, :])
    if table is None:
        return n
    t = _table_rows(table, indices, rows, sequence)
    shift = t[:, shift_slot * hidden:(shift_slot + 1) * hidden]
    scale = t[:, scale_slot * hidden:(scale_slot + 1) * hidden]
    return bf16_round(bf16_round(n * bf16_round(F32(1) + scale)) + shift)


def rms_adaln(x, weight, eps, table, indices, shift_slot, scale_slot, sequence=None,
              reduce=sumsq_tree):
    """RMSNorm + adaLN modulate, bf16 output (model/kernels.py:48-78, 260-272).

    x: [rows, hidden] float32 (bf16 values); row r uses table[indices[r % sequence]].
    """
    v = np.asarray(x, F32)
    seq = v.shape[0] if sequence is None else sequence
    return _rms_modulate(v, weight, eps, table, indices, seq, shift_slot, scale_slot, reduce)


def rms_adaln_quant_int8(x, weight, eps, table, indices, shift_slot, scale_slot, sequence=None,
                         reduce=sumsq_quant):
    """RMSNorm + adaLN modulate + per-row int8 quantisation
    (model/kernels.py:81-128, 275-289). Returns (int8, float32 [rows, 1])."""
    m = rms_adaln(x, weight, eps, table, indices, shift_slot, scale_slot, sequence, reduce)
    return quantize_rows(m)


def gated_residual(x, y, table, indices, gate_slot, sequence=None) -> np.ndarray:
    """bf16(x + bf16(gate * y)) (model/kernels.py:131-153, 292-304); table None -> gate 1."""
    x = np.asarray(x, F32)
    y = np.asarray(y, F32)
    rows, hidden = x.shape
    if table is None:
        gate = np.ones_like(x)
    else:
        seq = rows if sequence is None else sequence
        gate = _table_rows(table, indices, rows, seq)[:, gate_slot * hidden:(gate_slot + 1) * hidden]
    return bf16_round(x + bf16_round(gate * y))


def residual_rms_quant(x, update, weight, eps, table, indices, sequence=None, reduce=sumsq_quant):
    """Gated residual (slot 2) fused into the FFN prologue (slots 3, 4)
    (model/kernels.py:101-105, 405-419). Returns (residual, int8, float32 [rows,1])."""
    residual = gated_residual(x, update, table, indices, 2, sequence)
    q, s = rms_adaln_quant_int8(residual, weight, eps, table, indices, 3, 4, sequence, reduce)
    return residual, q, s


# ---------------------------------------------------------------- K6 / K7


def _silu_bf16(g):
    sig = (F32(1) / (F32(1) + np.exp(-g))).astype(F32)
    return bf16_round(g * sig)


def swiglu(projected) -> np.ndarray:
    """bf16(value * bf16(gate * sigmoid(gate))) over [rows, 2*inner]
    (model/kernels.py:156-166, 307-315)."""
    p = np.asarray(projected, F32)
    inner = p.shape[-1] // 2
    with np.errstate(over="ignore"):
        return bf16_round(p[..., :inner] * _silu_bf16(p[..., inner:]))


def swiglu_quant_int8(projected):
    """SwiGLU then per-row int8 quantisation (model/kernels.py:169-185, 318-328)."""
    return quantize_rows(swiglu(projected))


# --------------------------------------------- Q/K RMSNorm + RoPE (next row)


def _thread_butterflies(terms: np.ndarray) -> np.ndarray:
    """One term per thread over next_pow2(n) threads (missing terms zero): an
    xor butterfly over each 32-thread warp, then one over the warp sums."""
    rows, n = terms.shape
    block = 1 << max(0, (n - 1).bit_length())
    padded = np.zeros((rows, block), F32)
    padded[:, :n] = terms
    wt = min(32, block)
    lanes = padded.reshape(rows, block // wt, wt)
    idx = np.arange(wt)
    off = wt // 2
    while off:
        lanes = lanes + lanes[:, :, idx ^ off]
        off //= 2
    s = lanes[:, :, 0]
    off = s.shape[1] // 2
    while off:
        s = s[:, :off] + s[:, off:2 * off]
        off //= 2
    return s[:, 0]


def sumsq_qk(v: np.ndarray, rotary_dim: int) -> np.ndarray:
    """Head-row sum of squares in the order of the CUDA Q/K kernels, which is
    the order of the reference's compiled Q/K kernels (4 warps, one term per
    thread; exact for head dimensions up to 128):
      * full rotary (rotary_dim == width, width a multiple of 16), the paired
        kernel (model/kernels.py:217-222): terms x_i^2 + x_{i+width/2}^2 for
        i < width/2;
      * otherwise (model/kernels.py:374-375): terms x_i^2."""
    v = np.asarray(v, F32)
    rows, width = v.shape
    if rotary_dim == width and width % 16 == 0:
        half = width // 2
        return _thread_butterflies(v[:, :half] * v[:, :half] + v[:, half:] * v[:, half:])
    return _thread_butterflies(v * v)


def sumsq_qk_reference(v: np.ndarray, rotary_dim: int, ordered: bool) -> np.ndarray:
    """The reference Q/K kernels' sum order under the Triton interpreter:
    full-rotary kernel sums (left^2 + right^2) over the half block
    (model/kernels.py:217-222); the general kernel sums x^2 over the block
    (:374-375), or, ordered, ((s0 + s2) + (s1 + s3)) over 32-wide quarters
    (:332-343)."""
    v = np.asarray(v, F32)
    rows, width = v.shape
    if rotary_dim == width:
        half = width // 2
        block = 1 << max(0, (half - 1).bit_length())
        pair = np.zeros((rows, block), F32)
        pair[:, :half] = v[:, :half] * v[:, :half] + v[:, half:] * v[:, half:]
        return np.sum(pair, axis=-1, dtype=F32)
    if ordered:
        s = [np.sum(v[:, 32 * i:32 * (i + 1)] * v[:, 32 * i:32 * (i + 1)], axis=-1, dtype=F32) for i in range(4)]
        return (s[0] + s[2]) + (s[1] + s[3])
    block = 1 << max(0, (width - 1).bit_length())
    padded = np.zeros((rows, block), F32)
    padded[:, :width] = v
    return np.sum(padded * padded, axis=-1, dtype=F32)


def qk_norm_rope(x, weight, eps, cos, sin, rotary_dim, tokens, reduce=None):
    """Per-head RMSNorm + rotary embedding of one of Q or K
    (model/kernels.py:188-257 full rotary, :345-402 general).

    x: float32 [rows, head_dim] (bf16 values), one row per (batch, token, head);
    tokens: int [rows], the token of each row (its cos/sin row);
    cos, sin: float32 [sequence, rotary_dim]. Returns float32 [rows, head_dim]:
      n = bf16((x * r) * w), r = 1 / sqrt(sum x^2 / head_dim + eps)
      d < rotary_dim: bf16(bf16(n_d * c_d) + bf16(s_sign * n_pair * s_d)) with
      c, s the bf16-rounded tables, pair = d +- rotary_dim/2, sign - then +;
      d >= rotary_dim: n_d.
    """
    v = np.asarray(x, F32)
    rows, width = v.shape
    ss = sumsq_qk(v, rotary_dim) if reduce is None else reduce(v)
    r = (F32(1) / np.sqrt(ss / F32(width) + F32(eps))).astype(F32)
    n = bf16_round((v * r[:, None]) * np.asarray(weight, F32)[None, :])
    out = n.copy()
    half = rotary_dim // 2
    c = bf16_round(np.asarray(cos, F32)[tokens])
    s = bf16_round(np.asarray(sin, F32)[tokens])
    d = np.arange(rotary_dim)
    pair = np.where(d < half, d + half, d - half)
    sign = np.where(d < half, F32(-1), F32(1))
    rot = bf16_round(bf16_round(n[:, :rotary_dim] * c) + bf16_round((sign * n[:, pair]) * s))
    out[:, :rotary_dim] = rot
    return out


# ---------------------------------------------------------- W8A8 linear


def int8_linear_forward(x, weight_nk, weight_scale, bias=None) -> np.ndarray:
    """Int8Linear.forward torch path (model/int8.py:60-68, 41-58): quantise the
    rows, exact int32 GEMM with the [K, N] transpose view, bf16 epilogue."""
    q, s = quantize_rows(x)
    return int8_matmul(q, np.asarray(weight_nk, np.int8).T, s, np.asarray(weight_scale, F32).reshape(-1),
                       bias)


def quantize_weight(w):
    """Int8Linear(source) weight quantisation (model/int8.py:9-13): per output row."""
    return quantize_rows(np.asarray(w, F32))
