"""Packed Flash W8A8 checkpoint loading (lynnreal_omni_b200.flash_int8), on the CPU.

A small checkpoint in the release's layout (config, quantization config,
safetensors index and shards, checksums) is written to a temporary folder and
loaded with a stand-in transformer class: the quantised modules must become
Int8Linear layers from the packed tensors, every other tensor must load, the
Q/K/V concatenation must compute exactly the three separate projections, and
the checks must reject tampered metadata, shards and incomplete checkpoints
with the reference's messages (model/flash_int8.py:9-56).
"""
from __future__ import annotations

import hashlib
import json
from types import SimpleNamespace

import pytest
import torch
from torch import nn

from lynnreal_omni_b200 import flash_int8
from lynnreal_omni_b200.int8 import Int8Linear

safetensors_torch = pytest.importorskip("safetensors.torch")
D = 64


class _Attn(nn.Module):
    def __init__(self):
        super().__init__()
        self.to_q, self.to_k, self.to_v = nn.Linear(D, D), nn.Linear(D, D), nn.Linear(D, D, bias=False)
        self.to_out = nn.ModuleList([nn.Linear(D, D)])
        self.fused_projections = False


class _Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.attn = _Attn()
        self.scale_shift_table = nn.Parameter(torch.zeros(6, D))


class _Model(nn.Module):
    def __init__(self, layers):
        super().__init__()
        self.transformer_blocks = nn.ModuleList(_Block() for _ in range(layers))
        self.proj_out = nn.Linear(D, 8)


def _sha(path):
    return hashlib.sha256(path.read_bytes()).hexdigest()


def _write_checkpoint(folder, layers=2):
    g = torch.Generator().manual_seed(7)
    quantized = []
    tensors = {}
    for i in range(layers):
        for name in ("to_q", "to_k", "to_v", "to_out.0"):
            full = f"transformer_blocks.{i}.attn.{name}"
            quantized.append(full)
            tensors[full + ".weight_int8"] = torch.randint(-127, 128, (D, D), generator=g, dtype=torch.int8)
            tensors[full + ".weight_scale"] = torch.empty(D, 1).uniform_(0.5e-3, 2e-3, generator=g)
            if name != "to_v":
                tensors[full + ".bias"] = (0.02 * torch.randn(D, generator=g)).to(torch.bfloat16)
        tensors[f"transformer_blocks.{i}.scale_shift_table"] = torch.randn(6, D, generator=g)
    tensors["proj_out.weight"] = torch.randn(8, D, generator=g)
    tensors["proj_out.bias"] = torch.randn(8, generator=g)
    names = sorted(tensors)
    shards = {"model-00001-of-00002.safetensors": names[::2], "model-00002-of-00002.safetensors": names[1::2]}
    weight_map = {}
    for fname, keys in shards.items():
        safetensors_torch.save_file({k: tensors[k].contiguous() for k in keys}, str(folder / fname))
        weight_map.update({k: fname for k in keys})
    (folder / "config.json").write_text(json.dumps({"num_layers": layers}))
    (folder / "quantization_config.json").write_text(json.dumps({"quantized_modules": quantized}))
    (folder / "diffusion_pytorch_model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    checksums = {n: {"sha256": _sha(folder / n)} for n in
                 ("config.json", "quantization_config.json", "diffusion_pytorch_model.safetensors.index.json")}
    for fname in shards:
        checksums[fname] = {"sha256": _sha(folder / fname), "bytes": (folder / fname).stat().st_size}
    (folder / "checksums.json").write_text(json.dumps(checksums))
    return tensors


def _factory(config):
    return _Model(config["num_layers"])


def test_load_transformer_installs_packed_layers_and_fuses_qkv(tmp_path):
    tensors = _write_checkpoint(tmp_path)
    model = flash_int8.load_transformer(tmp_path, device="cpu", gemm="torch", model_factory=_factory)
    for i, block in enumerate(model.transformer_blocks):
        attn = block.attn
        assert attn.to_q is None and attn.to_k is None and attn.to_v is None and attn.fused_projections
        assert isinstance(attn.to_qkv, Int8Linear) and isinstance(attn.to_out[0], Int8Linear)
        # the fused QKV holds the Q, K, V rows, scales and biases in that order
        # (its projection then equals the three separate ones row for row)
        keys = [f"transformer_blocks.{i}.attn.{name}" for name in ("to_q", "to_k", "to_v")]
        rows = torch.cat([tensors[k + ".weight_int8"] for k in keys])
        scales = torch.cat([tensors[k + ".weight_scale"] for k in keys])
        assert torch.equal(attn.to_qkv.weight_int8.t(), rows)
        assert torch.equal(attn.to_qkv.weight_scale.t(), scales)
        biases = [tensors.get(k + ".bias") for k in keys]
        if any(b is not None for b in biases):
            expect = torch.cat([b if b is not None else torch.zeros(rows.shape[0] // 3, dtype=torch.bfloat16)
                                for b in biases])
            assert torch.equal(attn.to_qkv.bias, expect)
        assert torch.equal(block.scale_shift_table, tensors[f"transformer_blocks.{i}.scale_shift_table"])
    assert torch.equal(model.proj_out.weight, tensors["proj_out.weight"])
    assert not model.training


@pytest.mark.parametrize("tamper,message", [
    ("config.json", "Flash metadata checksum mismatch"),
    ("model-00002-of-00002.safetensors", "Flash shard checksum mismatch"),
])
def test_load_transformer_rejects_tampered_files(tmp_path, tamper, message):
    _write_checkpoint(tmp_path)
    with (tmp_path / tamper).open("ab") as f:
        f.write(b" ")
    with pytest.raises(ValueError, match=message):
        flash_int8.load_transformer(tmp_path, device="cpu", gemm="torch", model_factory=_factory)


def test_load_transformer_rejects_incomplete_checkpoint(tmp_path):
    _write_checkpoint(tmp_path)
    with pytest.raises(ValueError, match="Incomplete Flash model"):
        flash_int8.load_transformer(tmp_path, device="cpu", gemm="torch", model_factory=lambda c: _Model(3))


def test_fuse_qkv_without_biases():
    attn = SimpleNamespace(to_q=None, to_k=None, to_v=None, fused_projections=False)
    g = torch.Generator().manual_seed(3)
    parts = []
    for _ in range(3):
        w = torch.randint(-127, 128, (D, D), generator=g, dtype=torch.int8)
        s = torch.empty(D, 1).uniform_(0.5e-3, 2e-3, generator=g)
        parts.append(Int8Linear.from_packed(w, s, None, gemm="torch"))
    attn.to_q, attn.to_k, attn.to_v = parts
    flash_int8.fuse_qkv(SimpleNamespace(transformer_blocks=[SimpleNamespace(attn=attn)]), gemm="torch")
    assert attn.to_qkv.bias is None
    assert torch.equal(attn.to_qkv.weight_int8.t(), torch.cat([p.weight_int8.t() for p in parts]))
    assert torch.equal(attn.to_qkv.weight_scale, torch.cat([p.weight_scale for p in parts], dim=1))


@pytest.mark.gpu
def test_fused_qkv_projects_like_the_three_layers_on_gpu():
    """On the GPU the fused QKV layer's output equals the separate Q, K, V
    projections concatenated (model/flash_int8.py:47-55)."""
    attn = SimpleNamespace(to_q=None, to_k=None, to_v=None, fused_projections=False)
    g = torch.Generator().manual_seed(4)
    parts = []
    for with_bias in (True, False, True):
        w = torch.randint(-127, 128, (D, D), generator=g, dtype=torch.int8)
        s = torch.empty(D, 1).uniform_(0.5e-3, 2e-3, generator=g)
        b = (0.02 * torch.randn(D, generator=g)).to(torch.bfloat16) if with_bias else None
        parts.append(Int8Linear.from_packed(w.cuda(), s.cuda(), None if b is None else b.cuda(), gemm="torch"))
    attn.to_q, attn.to_k, attn.to_v = parts
    flash_int8.fuse_qkv(SimpleNamespace(transformer_blocks=[SimpleNamespace(attn=attn)]), gemm="torch")
    x = torch.randn(37, D, generator=g).to(torch.bfloat16).cuda()
    for fused in (False, True):
        for layer in parts + [attn.to_qkv]:
            layer.fused_ops = fused
        assert torch.equal(attn.to_qkv(x), torch.cat([p(x) for p in parts], dim=-1))
