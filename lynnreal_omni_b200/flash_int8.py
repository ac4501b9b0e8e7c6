"""Load the trained Flash W8A8 checkpoint without requantisation.

Replaces model/flash_int8.py:9-56 (``load_transformer``): the checkpoint's
metadata and shards are checked against ``checksums.json`` (SHA-256 and
sizes), every module named in ``quantization_config.json``
(``quantized_modules``) becomes an ``Int8Linear`` built from its packed
``.weight_int8`` / ``.weight_scale`` / ``.bias`` tensors, the remaining tensors
are loaded into the model as they are, and each block's Q, K and V
projections are concatenated into one ``to_qkv`` (integer rows and their
original per-channel scales, so the fused projection computes exactly the
three separate ones) — the layout ``fusion.FusedAttention`` consumes.

The transformer class itself belongs to diffusers (MiniMaxH3Transformer3DModel),
which this package does not ship: ``load_transformer`` builds it with
diffusers and accelerate when they are installed, or with a caller-supplied
``model_factory(config) -> nn.Module``.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch

from .int8 import Int8Linear

__all__ = ["load_transformer", "install_packed", "fuse_qkv", "sha256"]


def sha256(path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as f:
        for chunk in iter(lambda: f.read(8 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _default_factory(config):
    try:
        from accelerate import init_empty_weights
        from diffusers import MiniMaxH3Transformer3DModel
    except ImportError as e:  # the reference requires both as well
        raise ImportError("load_transformer needs diffusers and accelerate, or a model_factory") from e
    with init_empty_weights(include_buffers=False):
        return MiniMaxH3Transformer3DModel.from_config(config)


def _submodule(model, name):
    return model.get_submodule(name) if name else model


def install_packed(model, tensors: dict, quantized_modules, gemm: str = "triton") -> set:
    """Replace every module in ``quantized_modules`` with an ``Int8Linear``
    from its packed tensors (popped from ``tensors``); returns the names of the
    model's parameters those modules replaced."""
    replaced = set()
    for name in quantized_modules:
        weight = tensors.pop(name + ".weight_int8")
        scale = tensors.pop(name + ".weight_scale")
        bias = tensors.pop(name + ".bias", None)
        layer = Int8Linear.from_packed(weight, scale, bias, gemm)
        parent, _, key = name.rpartition(".")
        setattr(_submodule(model, parent), key, layer)
        replaced.update({name + ".weight", name + ".bias"})
    return replaced


def fuse_qkv(model, gemm: str = "triton") -> None:
    """Concatenate each block's quantised Q, K, V projections into ``to_qkv``
    (model/flash_int8.py:47-55): weight rows and their scales in Q, K, V
    order; a missing bias becomes zeros when any of the three has one."""
    for block in model.transformer_blocks:
        attn = block.attn
        parts = [attn.to_q, attn.to_k, attn.to_v]
        if any(p.bias is not None for p in parts):
            bias = torch.cat([p.bias if p.bias is not None else p.weight_int8.new_zeros(p.out_features,
                                                                                      dtype=torch.bfloat16)
                              for p in parts])
        else:
            bias = None
        attn.to_qkv = Int8Linear.from_packed(torch.cat([p.weight_int8.t() for p in parts]),
                                             torch.cat([p.weight_scale.t() for p in parts]), bias, gemm)
        attn.to_q = attn.to_k = attn.to_v = None
        attn.fused_projections = True


_METADATA = ("config.json", "quantization_config.json", "diffusion_pytorch_model.safetensors.index.json")


def _verified_metadata(folder: Path, checksums: dict) -> list:
    """The three metadata documents, each checked against its SHA-256 first."""
    docs = []
    for name in _METADATA:
        if sha256(folder / name) != checksums[name]["sha256"]:
            raise ValueError("Flash metadata checksum mismatch: " + name)
        docs.append(json.loads((folder / name).read_text()))
    return docs


def _verified_tensors(folder: Path, weight_map: dict, checksums: dict, device) -> dict:
    """All tensors of the checkpoint; every shard's size and SHA-256 are checked
    before it is read, and its tensor names against the index."""
    from safetensors.torch import load_file
    by_shard = {}
    for tensor_name, shard in weight_map.items():
        by_shard.setdefault(shard, set()).add(tensor_name)
    tensors = {}
    for shard in sorted(by_shard):
        path = folder / shard
        expect = checksums[shard]
        if path.stat().st_size != expect["bytes"] or sha256(path) != expect["sha256"]:
            raise ValueError("Flash shard checksum mismatch: " + shard)
        loaded = load_file(str(path), device=str(device))
        if set(loaded) != by_shard[shard]:
            raise ValueError("Flash shard index mismatch")
        tensors.update(loaded)
    return tensors


def load_transformer(folder, device="cuda", gemm="triton", model_factory=None):
    """Build the Flash transformer from a packed W8A8 checkpoint folder
    (model/flash_int8.py:9-56); same checks and error messages."""
    folder = Path(folder).resolve(strict=True)
    checksums = json.loads((folder / "checksums.json").read_text())
    config, quant, index = _verified_metadata(folder, checksums)
    model = (model_factory or _default_factory)(config)
    expected = set(model.state_dict())
    tensors = _verified_tensors(folder, index["weight_map"], checksums, device)
    expected -= install_packed(model, tensors, quant["quantized_modules"], gemm)
    if set(tensors) != expected:
        raise ValueError("Incomplete Flash model: " + str(set(tensors) ^ expected))
    result = model.load_state_dict(tensors, strict=False, assign=True)
    if result.unexpected_keys:
        raise ValueError(result.unexpected_keys)
    fuse_qkv(model, gemm)
    return model.to(device).eval().requires_grad_(False)
