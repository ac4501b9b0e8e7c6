"""The allocation-free GEMM entry point, lr_int8_gemm_noalloc.

It exists for callers that cannot allocate device memory when they run the
GEMM — a plugin or FFI host that only passes in the tensors it already owns,
or a framework whose memory pool is frozen during a step — so its split-K
scratch is a fixed array inside the library instead of a caller workspace.
These tests call it through the C ABI on shapes that do need that scratch and
check it against the allocating entry point, lr_int8_gemm, bit for bit (the
GEMM's tolerance everywhere in these tests), on two calls in a row so the
second call runs on the scratch the first one left behind. This file is
collected last on purpose.
"""
from __future__ import annotations

import pytest
import torch

from lynnreal_omni_b200 import _lib, workloads

pytestmark = pytest.mark.gpu
DEV = "cuda"
NOALLOC_SCRATCH_BYTES = 16 << 20  # LR_NOALLOC_SCRATCH_BYTES in include/lr_w8a8.h


def _gemm(name, a, b, rs, cs, bias, out, epilogue=_lib.LR_EPI_NONE, resid=None, table=None, idx=None,
          gate_slot=0):
    """Call one GEMM entry point of the C ABI on caller-owned CUDA tensors."""
    lib = _lib.load()
    m, k = a.shape
    n = b.shape[1]
    seq = m
    st = getattr(lib, name)(
        a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), b.stride(1), m, n, k, rs.data_ptr(),
        cs.data_ptr(), None if bias is None else bias.data_ptr(), epilogue,
        None if resid is None else resid.data_ptr(), 0 if resid is None else resid.stride(0),
        None if table is None else table.data_ptr(), 0 if table is None else table.shape[0],
        0 if table is None else table.shape[1], None if idx is None else idx.data_ptr(), seq, gate_slot,
        out.data_ptr(), out.stride(0), torch.cuda.current_stream().cuda_stream)
    return st


def _operands(m, k, n, seed):
    a, b, rs, cs, bias = workloads.gemm_operands(m, k, n, seed=seed, bias=True)
    return (a.to(DEV), b.to(DEV), rs.to(DEV).reshape(-1).contiguous(), cs.to(DEV).reshape(-1).contiguous(),
            bias.to(DEV))


def test_noalloc_matches_lr_int8_gemm_on_two_calls_in_a_row():
    lib = _lib.load()
    # call 1: plain epilogue, 9 MiB of split-K scratch
    m, k, n = 128, 6144, 6144
    need = lib.lr_int8_gemm_workspace_bytes(m, n, k)
    assert 0 < need <= NOALLOC_SCRATCH_BYTES
    a, b, rs, cs, bias = _operands(m, k, n, seed=31)
    ref = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    got = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    _lib.check(_gemm("lr_int8_gemm", a, b, rs, cs, bias, ref), "lr_int8_gemm")
    _lib.check(_gemm("lr_int8_gemm_noalloc", a, b, rs, cs, bias, got), "lr_int8_gemm_noalloc")
    torch.cuda.synchronize()
    assert torch.equal(got, ref)

    # call 2: another shape and the gated-residual epilogue, on the scratch the
    # first call left behind
    m, k, n = 64, 24576, 6144
    assert 0 < lib.lr_int8_gemm_workspace_bytes(m, n, k) <= NOALLOC_SCRATCH_BYTES
    a, b, rs, cs, bias = _operands(m, k, n, seed=32)
    gen = torch.Generator().manual_seed(32)
    resid = torch.randn(m, n, generator=gen).to(torch.bfloat16).to(DEV)
    table = (0.3 * torch.randn(2, 6 * n, generator=gen)).to(torch.bfloat16).to(DEV)
    idx = torch.randint(0, 2, (m,), generator=gen).to(DEV)
    ref = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    got = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    kw = dict(epilogue=_lib.LR_EPI_GATED_RESIDUAL, resid=resid, table=table, idx=idx, gate_slot=5)
    _lib.check(_gemm("lr_int8_gemm", a, b, rs, cs, bias, ref, **kw), "lr_int8_gemm")
    _lib.check(_gemm("lr_int8_gemm_noalloc", a, b, rs, cs, bias, got, **kw), "lr_int8_gemm_noalloc")
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    assert _lib.device_status(clear=True) == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """A shape whose split-K scratch would exceed the 16 MiB array is refused
    with a clear error instead of running."""
    lib = _lib.load()
    m, k, n = 256, 6144, 6144
    assert lib.lr_int8_gemm_workspace_bytes(m, n, k) > NOALLOC_SCRATCH_BYTES
    a, b, rs, cs, bias = _operands(m, k, n, seed=33)
    out = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    st = _gemm("lr_int8_gemm_noalloc", a, b, rs, cs, bias, out)
    assert st == _lib.LR_ERR_UNSUPPORTED
    assert b"static maximum" in lib.lr_last_error()


def test_noalloc_calls_leave_free_device_memory_unchanged():
    """After a first call (which may load the library's GPU code, and with it
    the scratch array, under CUDA's lazy module loading), further calls change
    the device's free memory by nothing: they allocate nothing."""
    lib = _lib.load()
    m, k, n = 128, 6144, 6144
    assert lib.lr_int8_gemm_workspace_bytes(m, n, k) > 0  # takes the split-K scratch
    a, b, rs, cs, bias = _operands(m, k, n, seed=34)
    out = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    _lib.check(_gemm("lr_int8_gemm_noalloc", a, b, rs, cs, bias, out), "lr_int8_gemm_noalloc")
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        _lib.check(_gemm("lr_int8_gemm_noalloc", a, b, rs, cs, bias, out), "lr_int8_gemm_noalloc")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    assert _lib.device_status(clear=True) == 0
