"""TMA-fed INT8 GEMM entry point (replaces model/int8_tma.py).

The reference's module is a Hopper-only persistent TMA kernel with a stricter
contract than ``int8_matmul``. On B200 every tensor-core launch of
``int8_matmul`` is already a persistent TMA kernel, so ``matmul`` keeps the
reference's signature and contract check and runs the same sm_100a kernel.
"""
from __future__ import annotations

import torch

from .int8_gemm import _launch
from . import _lib


def matmul(a, b, sa, sb, bias=None, tile=(128, 256, 128, 8, 3)):
    """bf16((a @ b) * sa * sb + bias); model/int8_tma.py:32-41.

    Requires row-major int8 activations and the transposed row-major weight view
    (``b.stride() == (1, K)``), else ValueError (model/int8_tma.py:34-35).
    """
    m, k = a.shape
    if a.dtype != torch.int8 or b.dtype != torch.int8 or not a.is_contiguous() or b.stride() != (1, k):
        raise ValueError("TMA requires row-major INT8 activations and transposed row-major weights")
    return _launch(a, b, sa, sb, bias, _lib.LR_EPI_NONE)
