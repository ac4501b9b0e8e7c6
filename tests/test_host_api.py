"""CPU tests of the C ABI library and of the host-side API (no GPU needed)."""
from __future__ import annotations

import ctypes
import json
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch
from torch import nn

from lynnreal_omni_b200 import _lib
from lynnreal_omni_b200.int8 import Int8Linear, quantize_transformer

ROOT = Path(__file__).resolve().parents[1]


def test_library_exports_every_declared_symbol():
    declared = _lib.header_symbols()
    assert len(declared) >= 12
    lib = _lib.load()
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    assert set(declared) == set(_lib.SIGNATURES), "binding and header disagree"


def test_library_version_and_error_path_without_gpu():
    lib = _lib.load()
    assert lib.lr_version() >= 100
    # argument validation happens on the host, before any CUDA call
    st = lib.lr_quantize_rows(None, 4, 0, 0, None, None, None)
    assert st == _lib.LR_ERR_INVALID_ARGUMENT
    assert b"invalid shape" in lib.lr_last_error()
    st = lib.lr_int8_gemm(None, 4, None, 1, 8, 4, 8, 16, None, None, None, 0, None, 0, None, 0, 0, None, 1, 0,
                          None, 8, None)
    assert st == _lib.LR_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _lib.check(st, "int8_matmul")


def test_workspace_query():
    """Split-K needs an M*N int32 workspace only when the output tiles cannot
    fill the GPU (small M); large shapes need none."""
    lib = _lib.load()
    assert lib.lr_int8_gemm_workspace_bytes(256, 6144, 6144) == 3 * 256 * 6144 * 4  # 3 K slices
    assert lib.lr_int8_gemm_workspace_bytes(12240, 24576, 6144) == 0
    assert lib.lr_int8_gemm_workspace_bytes(256, 6144, 512) == 0  # too little K to split
    assert lib.lr_int8_gemm_workspace_bytes(0, 6144, 6144) == 0


def test_empty_rows_are_a_no_op():
    lib = _lib.load()
    assert lib.lr_quantize_rows(None, 0, 64, 64, None, None, None) == _lib.LR_OK
    assert lib.lr_gated_residual(None, None, None, 0, 0, None, 1, 0, 64, 0, None, None) == _lib.LR_OK


def test_ops_refuse_cpu_tensors():
    """No CPU path behind the product functions: host tensors are an error."""
    from types import SimpleNamespace
    from lynnreal_omni_b200 import kernels as K, flash
    from lynnreal_omni_b200.attention import attention_bshd
    with pytest.raises(ValueError):
        K.quantize_rows(torch.zeros(2, 8, dtype=torch.bfloat16))
    x = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        attention_bshd(x, x, x)
    norm = SimpleNamespace(weight=torch.ones(128, dtype=torch.bfloat16), eps=1e-6)
    with pytest.raises(ValueError):
        K.qk_norm_rope(x, x, norm, norm, (torch.ones(4, 128), torch.zeros(4, 128)))
    with pytest.raises(ValueError):
        flash.index_select(torch.zeros(4, 8), 0, torch.tensor([1, 2]))
    h = torch.zeros(1, 4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        flash.restore(h, h, h, torch.zeros(4, dtype=torch.int64))
    with pytest.raises(ValueError):
        flash.spatial_layout(torch.zeros(4, 3), torch.zeros(4, dtype=torch.int64))


def test_empty_and_degenerate_calls_are_no_ops():
    lib = _lib.load()
    assert lib.lr_gather_rows(None, 0, 0, 0, 0, None, 0, None, 0, None) == _lib.LR_OK
    assert lib.lr_flash_restore(None, None, None, None, 0, 0, 0, 0, 1.0, None, None) == _lib.LR_OK
    assert lib.lr_flash_nearest_anchor(None, 0, None, 0, None, 0, None, None) == _lib.LR_OK
    assert lib.lr_attention_bf16(None, 128, None, 128, None, 128, 0, 0, 0, 1, 128, 1.0, None, 128, None) == _lib.LR_OK
    assert lib.lr_attention_bf16(None, 128, None, 128, None, 128, 1, 4, 4, 1, 64, 1.0, None, 128, None) == \
        _lib.LR_ERR_UNSUPPORTED


def test_int8_linear_contract():
    with pytest.raises(ValueError):
        Int8Linear(nn.Linear(8, 4), gemm="cublas")
    with pytest.raises(ValueError):
        Int8Linear.from_packed(torch.zeros(4, 8), torch.ones(4, 1))
    with pytest.raises(ValueError):
        Int8Linear.from_packed(torch.zeros(4, 8, dtype=torch.int8), torch.ones(4))
    layer = Int8Linear.from_packed(torch.zeros(4, 8, dtype=torch.int8), torch.ones(4, 1))
    assert layer.in_features == 8 and layer.out_features == 4 and layer.gemm == "triton"
    assert layer.weight_int8.shape == (8, 4) and layer.weight_int8.stride() == (1, 8)
    assert layer.weight.dtype == torch.bfloat16 and layer.weight.numel() == 0
    assert not layer.fused_ops


def test_int8_linear_has_no_cpu_path():
    """Every backend name runs the sm_100a kernels; a CPU tensor is refused
    instead of being computed by another implementation."""
    from lynnreal_omni_b200 import workloads
    x, pl = workloads.config0(seed=8, m=21, k=256, n=72)
    for gemm in ("torch", "triton", "b200"):
        layer = Int8Linear.from_packed(pl.weight, pl.scale, pl.bias, gemm=gemm)
        for fused in (False, True):
            layer.fused_ops = fused
            with pytest.raises(ValueError):
                layer(x.view(1, 21, 256))


def test_int8_linear_weight_quantisation_matches_reference_golden():
    """Int8Linear(nn.Linear) stores the reference's int8 rows and scales
    (golden vectors of model/int8.py:7-20 run on the CPU)."""
    import numpy as np
    from oracle import w8a8_oracle as O
    data = np.load(ROOT / "tests" / "golden" / "w8a8_small.npz")
    w = torch.from_numpy(O.from_bf16_bits(data["wq.w"])).to(torch.bfloat16)
    src = nn.Linear(w.shape[1], w.shape[0], bias=False).to(torch.bfloat16)
    with torch.no_grad():
        src.weight.copy_(w)
    layer = Int8Linear(src, gemm="torch")
    np.testing.assert_array_equal(layer.weight_int8.t().contiguous().numpy(), data["wq.q"])
    np.testing.assert_array_equal(layer.weight_scale.t().contiguous().numpy(), data["wq.s"])
    assert layer.weight_int8.stride() == (1, w.shape[1]) and layer.weight.dtype == torch.bfloat16


class _Attn(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.to_q, self.to_k, self.to_v = nn.Linear(d, d), nn.Linear(d, d), nn.Linear(d, d, bias=False)
        self.to_out = nn.ModuleList([nn.Linear(d, d), nn.Dropout(0.0)])


class _Proj(nn.Module):
    def __init__(self, d, f):
        super().__init__()
        self.proj = nn.Linear(d, f)


class _Block(nn.Module):
    def __init__(self, d, f):
        super().__init__()
        self.attn = _Attn(d)
        self.ff = SimpleNamespace(net=nn.ModuleList([_Proj(d, f), nn.Dropout(0.0), nn.Linear(f, d)]))


def test_quantize_transformer_matches_reference_report():
    golden = json.loads((ROOT / "tests" / "golden" / "quantize_transformer.json").read_text())
    torch.manual_seed(5)
    model = SimpleNamespace(transformer_blocks=[_Block(32, 64) for _ in range(4)])
    report = quantize_transformer(model, protected_edges=1, gemm="torch")
    assert report == golden
    b1 = model.transformer_blocks[1]
    assert isinstance(b1.attn.to_qkv, Int8Linear) and b1.attn.to_qkv.out_features == 96
    assert isinstance(model.transformer_blocks[0].attn.to_qkv, nn.Linear)
    with pytest.raises(ValueError):
        quantize_transformer(SimpleNamespace(transformer_blocks=[_Block(8, 8)]), protected_edges=1)


def test_c_header_compiles_as_c():
    """include/lr_w8a8.h is plain C."""
    import subprocess
    import tempfile
    src = '#include "lr_w8a8.h"\nint main(void){ return lr_version() < 0; }\n'
    with tempfile.TemporaryDirectory() as d:
        c = Path(d) / "t.c"
        c.write_text(src)
        r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-I", str(ROOT / "include"),
                            str(c)], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_arithmetic_mode_rejects_unknown_modes_without_a_gpu():
    """lr_set_arithmetic validates its argument on the host, before any CUDA
    call; the Python wrapper refuses names it does not know."""
    lib = _lib.load()
    assert lib.lr_set_arithmetic(7) == _lib.LR_ERR_INVALID_ARGUMENT
    assert b"unknown mode" in lib.lr_last_error()
    assert lib.lr_get_arithmetic(None) == _lib.LR_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _lib.set_arithmetic("fast")
