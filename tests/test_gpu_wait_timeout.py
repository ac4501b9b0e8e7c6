"""The GEMM's bounded waits, made to run out on purpose (no GPU fault).

Every mbarrier wait of the tensor-core GEMM gives up after a limit, raises
device status bit 1, drains its own copies and tensor-core work, frees its
tensor memory and returns (lynnreal_omni_b200/csrc/lr_gemm_sm100.cu,
wait_bounded). Here the test hook lr_gemm_test_wait shortens the limit to
1 ms and makes one launch skip a TMA load, so one stage's barrier never
completes: the call must return within a few limits, report the timeout bit,
and leave the context usable, with the next GEMM on the same stream exact.
The reference has no such path; its analogue is the recoverable-failure
classification of model/acceleration.py:49-56.
"""
from __future__ import annotations

import time

import pytest
import torch

from lynnreal_omni_b200 import _lib, workloads
from lynnreal_omni_b200.int8_gemm import int8_matmul

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIMEOUT_BIT = 2


def test_gemm_wait_runs_out_reports_and_recovers():
    lib = _lib.load()
    # 512 x 256 -> 512: four 256 x 256 tiles on the CTA-pair kernel, K too
    # short to split
    a, b, rs, cs, bias = workloads.gemm_operands(512, 256, 512, seed=4, device=DEV, bias=True)
    good = int8_matmul(a, b, rs, cs, bias)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    _lib.check(lib.lr_gemm_test_wait(1_000_000, 1), "gemm_test_wait")  # 1 ms, drop one load
    try:
        t0 = time.monotonic()
        int8_matmul(a, b, rs, cs, bias)  # one stage of cluster 0 never completes
        torch.cuda.synchronize()
        elapsed = time.monotonic() - t0
        status = _lib.device_status(clear=True)
    finally:
        _lib.check(lib.lr_gemm_test_wait(0, 0), "gemm_test_wait")
    assert status & TIMEOUT_BIT, status
    assert elapsed < 5.0, elapsed
    # the next launches run normally and exactly
    for _ in range(2):
        assert torch.equal(int8_matmul(a, b, rs, cs, bias), good)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0


def test_gemm_test_hook_validates_its_limit():
    lib = _lib.load()
    assert lib.lr_gemm_test_wait(-1, 0) == _lib.LR_ERR_INVALID_ARGUMENT
