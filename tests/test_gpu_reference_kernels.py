"""The kernels against the reference's own compiled kernels on the same GPU.

The reference installed into ``baseline/_ref`` (``pip install --no-deps
--target baseline/_ref <reference>``) is imported and its Triton kernels run
on this B200 next to this package's, on the same seeded inputs. In the default
arithmetic mode the int8 activations, row scales and bf16 outputs are bit-exact
against them: the reference's compiled kernels divide with div.full.f32 and
take tl.rsqrt as rsqrt.approx.f32, and their tl.sum over 8 warps adds each
thread's 8-column chunks in order, then by xor butterflies within and across
warps; the kernels here do the same. The reference's INT8 GEMM kernel does not
compile under this image's Triton, so its int8_matmul runs its own PyTorch
path, which the GEMM here reproduces exactly. Skipped where the reference is
not installed.
"""
from __future__ import annotations

import json
import sys
import warnings
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

from lynnreal_omni_b200 import _lib, kernels as K
from lynnreal_omni_b200.int8_gemm import int8_matmul

pytestmark = [pytest.mark.gpu, pytest.mark.reference_gpu_arith]
DEV = "cuda"
REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def ref():
    if not (REF / "lynnreal" / "model" / "kernels.py").exists():
        pytest.skip("the reference is not installed in baseline/_ref")
    sys.path.insert(0, str(REF))
    try:
        import lynnreal.model.int8_gemm as rg
        import lynnreal.model.kernels as rk
    except Exception as error:  # triton or torch mismatch in this image
        pytest.skip(f"the installed reference does not import: {error}")
    finally:
        sys.path.remove(str(REF))
    return SimpleNamespace(kernels=rk, gemm=rg)


def same(a, b):
    assert a.shape == b.shape and a.dtype == b.dtype
    if not torch.equal(a, b):
        diff = (a.view(torch.int8 if a.element_size() == 1 else torch.int16).int()
                - b.view(torch.int8 if b.element_size() == 1 else torch.int16).int()).abs() if a.element_size() <= 2 \
            else (a.view(torch.int32) - b.view(torch.int32)).abs()
        raise AssertionError(f"{int((diff != 0).sum())} of {a.numel()} differ, max bit distance {int(diff.max())}")


def inputs(m, d, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(1, m, d, device=DEV, generator=g).bfloat16()
    y = torch.randn(1, m, d, device=DEV, generator=g).bfloat16()
    norm = SimpleNamespace(weight=(1 + 0.05 * torch.randn(d, device=DEV, generator=g)).bfloat16(), eps=1e-6)
    table = (0.1 * torch.randn(3, 6 * d, device=DEV, generator=g)).bfloat16()
    idx = torch.randint(0, 3, (m,), device=DEV, generator=g)
    return x, y, norm, table, idx


@pytest.mark.parametrize("m,d", [(2048, 6144), (1531, 5376), (512, 24576), (300, 4096)])
def test_row_kernels_equal_the_compiled_reference(ref, m, d):
    assert _lib.arithmetic() == "reference_gpu"
    rk = ref.kernels
    x, y, norm, table, idx = inputs(m, d, seed=m + d)
    for got, want in zip(K.quantize_rows(x.view(m, d)), rk.quantize_rows(x.view(m, d))):
        same(got, want)
    for slots in ((0, 1), (3, 4)):
        for got, want in zip(K._rms_adaln_quant_int8(x, norm, table, idx, *slots),
                             rk._rms_adaln_quant_int8(x, norm, table, idx, *slots)):
            same(got, want)
        same(K._rms_adaln(x, norm, table, idx, *slots), rk._rms_adaln(x, norm, table, idx, *slots))
    for got, want in zip(K.residual_rms_quant(x, y, norm, table, idx), rk.residual_rms_quant(x, y, norm, table, idx)):
        same(got, want)
    same(K._gated_residual(x, y, table, idx, 2), rk._gated_residual(x, y, table, idx, 2))
    assert _lib.device_status(clear=True) == 0


@pytest.mark.parametrize("m,inner", [(1024, 14336), (777, 12288), (64, 2688)])
def test_swiglu_equals_the_compiled_reference(ref, m, inner):
    rk = ref.kernels
    g = torch.Generator(device=DEV).manual_seed(inner)
    p = (2 * torch.randn(m, 2 * inner, device=DEV, generator=g)).bfloat16()
    same(K._swiglu(p), rk._swiglu(p))
    for got, want in zip(K._swiglu_quant_int8(p), rk._swiglu_quant_int8(p)):
        same(got, want)


@pytest.mark.parametrize("m,k,n", [(2048, 6144, 6144), (256, 6144, 6144), (1000, 4096, 5376)])
def test_gemm_equals_the_reference(ref, m, k, n):
    g = torch.Generator(device=DEV).manual_seed(m + k + n)
    a = torch.randint(-127, 128, (m, k), generator=g, device=DEV, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, device=DEV, dtype=torch.int8).t()
    rs = torch.rand(m, 1, generator=g, device=DEV) / 127
    cs = torch.rand(1, n, generator=g, device=DEV) / 127
    bias = (0.02 * torch.randn(n, generator=g, device=DEV)).bfloat16()
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")  # the reference reports its fallback to its torch path
        want = ref.gemm.int8_matmul(a, b, rs, cs, bias)
    same(int8_matmul(a, b, rs, cs, bias), want)


def test_ieee_mode_differs_only_in_rounding(ref):
    """The oracle's IEEE mode and the default mode agree except for the rare
    quotients that div.full.f32 rounds differently (one int8 step)."""
    m, d = 1024, 6144
    x, _, norm, table, idx = inputs(m, d, seed=9)
    default = K._rms_adaln_quant_int8(x, norm, table, idx, 0, 1)
    _lib.set_arithmetic("ieee")
    try:
        ieee = K._rms_adaln_quant_int8(x, norm, table, idx, 0, 1)
    finally:
        _lib.set_arithmetic("reference_gpu")
    step = (default[0].int() - ieee[0].int()).abs()
    assert int(step.max()) <= 1 and float((step != 0).float().mean()) < 1e-3


def test_outputs_equal_the_recorded_reference_outputs():
    """Same comparison without the installed reference: SHA-256 digests of the
    reference's compiled kernels' outputs on a B200, recorded by
    tests/golden/make_reference_gpu.py on seeded inputs it regenerates."""
    path = Path(__file__).resolve().parent / "golden" / "reference_gpu.json"
    if not path.exists():
        pytest.skip("no recorded reference outputs")
    sys.path.insert(0, str(path.parent))
    try:
        import make_reference_gpu as R
    finally:
        sys.path.remove(str(path.parent))
    record = json.loads(path.read_text())
    assert _lib.arithmetic() == "reference_gpu"
    checked = 0
    for name, case in record["cases"].items():
        inp = R.reference_gpu_inputs(case["rows"], case["width"], case["seed"], DEV)
        ours = R.outputs(K, name.split("_")[0], inp)
        for key, digests in case["sha256"].items():
            got = [R.digest(t) for t in ours[key]]
            assert got == digests, (name, key)
            checked += len(digests)
    for name, case in record.get("qk", {}).items():
        inp = R.qk_inputs(case["tokens"], case["heads"], case["head_dim"], case["rotary_dim"], case["seed"], DEV)
        got = K.qk_norm_rope(inp.q, inp.k, inp.norm_q, inp.norm_k, (inp.cos, inp.sin))
        assert [R.digest(t) for t in got] == case["sha256"], name
        checked += 2
    assert checked >= 30


@pytest.mark.parametrize("s,h,d,rot", [(2048, 48, 128, 128), (1000, 16, 128, 64), (1025, 8, 96, 96),
                                       (700, 8, 64, 32)])
def test_qk_norm_rope_equals_the_compiled_reference(ref, s, h, d, rot):
    """Q/K RMSNorm + RoPE on strided views of one fused QKV output, launched
    for the reference the way its FusedAttention does (model/fusion.py:29-54;
    on B200 without the ordered reduction, which it enables only on Hopper)."""
    import triton
    rk = ref.kernels
    g = torch.Generator(device=DEV).manual_seed(s + d + rot)
    qkv = torch.randn(1, s, 3 * h * d, device=DEV, generator=g).bfloat16()
    q, k, _ = [t.unflatten(-1, (h, -1)) for t in qkv.chunk(3, dim=-1)]
    nq = SimpleNamespace(weight=(1 + 0.05 * torch.randn(d, device=DEV, generator=g)).bfloat16(), eps=1e-6)
    nk = SimpleNamespace(weight=(1 + 0.05 * torch.randn(d, device=DEV, generator=g)).bfloat16(), eps=1e-6)
    phase = torch.randn(s, rot, device=DEV, generator=g)
    cos, sin = phase.cos(), phase.sin()
    q_out = torch.empty_like(q, memory_format=torch.contiguous_format)
    k_out = torch.empty_like(k, memory_format=torch.contiguous_format)
    common = (q, k, nq.weight, nk.weight, cos, sin, q_out, k_out, s, h, q.stride(1), q.stride(2),
              k.stride(1), k.stride(2), d)
    grid = (q.numel() // d,)
    if rot == d:
        rk._qk_norm_full_rope_paired_kernel[grid](*common, float(nq.eps), triton.next_power_of_2(d // 2),
                                                 num_warps=4, enable_fp_fusion=False)
    else:
        rk._qk_norm_rope_kernel[grid](*common, rot, float(nq.eps), triton.next_power_of_2(d), num_warps=4,
                                      enable_fp_fusion=False)
    oq, ok = K.qk_norm_rope(q, k, nq, nk, (cos, sin))
    same(oq, q_out)
    same(ok, k_out)
